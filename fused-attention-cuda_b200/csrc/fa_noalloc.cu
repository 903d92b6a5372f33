// fa_noalloc.cu -- fa_forward without a caller-provided workspace: the scratch the fp32 path
// needs (tf32-rounded copies of q, k, v) comes from a fixed device array compiled into this
// library, so a call performs no allocation.  It is for callers that cannot allocate device
// memory when they call: runtimes that reserve all device memory up front and hand a plugin no
// allocator, and latency-critical loops that avoid cudaMalloc/cudaFree because those can
// synchronize the device.  fp16/bf16 need no scratch and go straight to fa_forward.
//
// The scratch is one array per CUDA context, shared by every call in that context: two calls
// whose executions overlap on the device (different streams, or different host threads) race on
// it.  Nothing in it has to start at zero: the rounding pre-pass writes every byte the attention
// kernel reads before it reads it.
//
// Its device address is looked up on every call that needs it (cudaGetSymbolAddress, with the
// caller's device and context current), not cached: an address belongs to a context, and a
// remembered one would be stale after cudaDeviceReset or in a context the caller created itself.
// The lookup allocates nothing, except once: under CUDA's default lazy module loading, the first
// lookup in a context loads this file's module, and with it the array.  Make one fp32 call (a
// tiny one will do) in each context before reserving the rest of device memory and before any
// stream capture.
#include <cuda_runtime.h>

#include <cstddef>

#include "fa_launch.h"
#include "fa_sm100.h"

namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[FA_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array in the current context.
cudaError_t scratch_in_current_context(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  *out = p;
  return cudaSuccess;
}

}  // namespace

extern "C" size_t fa_noalloc_scratch_bytes(void) { return FA_NOALLOC_SCRATCH_BYTES; }

extern "C" int fa_forward_noalloc(int impl, int dtype, const void* q, const void* k,
                                  const void* v, void* o, float* lse, const fa_params_t* p,
                                  cudaStream_t stream) {
  const size_t need = fa_workspace_bytes(impl, dtype, p);
  if (need == 0) return fa_forward(impl, dtype, q, k, v, o, lse, nullptr, p, stream);
  // The same checks and error codes as fa_forward, before the module is touched.
  if (const cudaError_t e = fa_sm100::check_forward_args(impl, dtype, q, k, v, o, lse, nullptr,
                                                         false, p, nullptr)) {
    return static_cast<int>(e);
  }
  if (need > FA_NOALLOC_SCRATCH_BYTES) return cudaErrorInvalidValue;
  void* scratch = nullptr;
  const cudaError_t e = scratch_in_current_context(&scratch);
  if (e != cudaSuccess) return static_cast<int>(e);
  return fa_forward(impl, dtype, q, k, v, o, lse, scratch, p, stream);
}
