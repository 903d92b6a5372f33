// fa_noalloc.cu -- fa_forward without a caller-provided workspace: the scratch the fp32 path
// needs (tf32-rounded copies of q, k, v) comes from a fixed device array compiled into this
// library, so the call performs no allocation of any kind.  It is for callers that cannot
// allocate device memory when they call: a host function enqueued on a stream may make no CUDA
// API calls at all, some runtimes reserve all device memory up front and hand a plugin no
// allocator, and latency-critical loops avoid cudaMalloc/cudaFree because they can synchronize
// the device.  fp16/bf16 need no scratch and go straight to fa_forward.
//
// The scratch is one array per device context, shared by every call: two calls whose lifetimes
// overlap on the device (different streams, or different host threads) race on it.  Its device
// address is looked up (cudaGetSymbolAddress) on the first call for each device; that first call
// should happen before any stream capture.  Nothing in it has to start at zero: the rounding
// pre-pass writes every byte the attention kernel reads before it reads it.
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>

#include "fa_sm100.h"

namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[FA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_ptr[kMaxDevices];

// Device address of the scratch array on the current device, looked up once per device.
cudaError_t scratch_on_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev].store(p, std::memory_order_release);
  }
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
  if (need > FA_NOALLOC_SCRATCH_BYTES) return cudaErrorInvalidValue;
  void* scratch = nullptr;
  const cudaError_t e = scratch_on_current_device(&scratch);
  if (e != cudaSuccess) return static_cast<int>(e);
  return fa_forward(impl, dtype, q, k, v, o, lse, scratch, p, stream);
}
