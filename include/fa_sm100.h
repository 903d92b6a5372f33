/* fa_sm100.h -- C ABI of the B200 (sm_100a) fused SDPA forward.
 *
 * This is the drop-in boundary.  Every entry point replaces one function of the reference's
 * frozen C++ kernel API, include/fa/attention.cuh (yashpatil582/fused-attention-cuda), with
 * the same argument meaning, the same layout contract and the same error convention, flattened
 * to `extern "C"` with plain pointers, ints and a POD struct so that ctypes / cgo / JNI / N-API
 * can bind it without C++ name mangling or torch types.
 *
 * Layout contract (attention.cuh:38-40): q, o are [B, H, N, D]; k, v are [B, Hkv, N, D]; all
 * contiguous with D fastest, 16-byte aligned; lse is [B, H, N] fp32, natural-log logsumexp of
 * the scaled scores per query row (m*scale + ln l; +inf for a row that sees no key).
 * Causal masks are top-left aligned (key j visible to query i iff j <= i), Nq == Nkv.
 *
 * Error convention (attention.cuh:43-45, src/dispatch.cu:96-111): functions return a
 * cudaError_t value as int and never abort; cudaErrorInvalidValue (1) for bad parameters,
 * cudaErrorNotSupported (801) when (impl, dtype, D, device) is not built.  Launches are
 * asynchronous on the caller's stream and never synchronise.  Messages go to stderr only when
 * FA_VERBOSE is set.  Device-side bounded waits report through fa_last_device_error().
 *
 * Threading: the debug overrides and the wait-time limit are process-global and not
 * thread-safe (as g_overrides in src/dispatch.cu:136).
 */
#ifndef FA_SM100_H_
#define FA_SM100_H_

#include <cuda_runtime_api.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element type of q/k/v/o -- fa::Dtype (attention.cuh:17). */
enum fa_dtype { FA_DTYPE_F32 = 0, FA_DTYPE_F16 = 1, FA_DTYPE_BF16 = 2 };

/* Implementation id -- fa::Impl (attention.cuh:20-26).  This build implements FA_IMPL_TUNED
 * (fp16/bf16) and FA_IMPL_FUSED (fp32 on tf32 tensor cores, and fp16), both on the one
 * tcgen05/TMA kernel; the reference's teaching rungs 1, 2 and 4 report cudaErrorNotSupported. */
enum fa_impl {
  FA_IMPL_NAIVE = 1,
  FA_IMPL_TILED = 2,
  FA_IMPL_FUSED = 3,
  FA_IMPL_WMMA = 4,
  FA_IMPL_TUNED = 5
};

/* fa::Params (attention.cuh:28-36); `causal` is an int instead of a C++ bool. */
typedef struct fa_params {
  int B;       /* batch */
  int H;       /* query heads */
  int Hkv;     /* key/value heads, H % Hkv == 0 */
  int N;       /* sequence length (Nq == Nkv), N % 32 == 0 */
  int D;       /* head dim, 64 or 128 */
  float scale; /* softmax scale, finite and > 0 (PyTorch default 1/sqrt(D)) */
  int causal;  /* 0/1, top-left aligned */
} fa_params_t;

/* fa::forward (attention.cuh:46-47; implementation src/dispatch.cu:140-161).
 * Launches the fused forward on `stream`.  `workspace` (caller-owned, 16-byte aligned) must hold
 * fa_workspace_bytes(impl, dtype, p) bytes; it may be NULL when that is 0.  The kernel reads
 * q, k, v and writes only o, lse and the workspace. */
int fa_forward(int impl, int dtype, const void* q, const void* k, const void* v, void* o,
               float* lse, void* workspace, const fa_params_t* p, cudaStream_t stream);

/* No counterpart in the reference (whose API takes contiguous tensors only): element strides of
 * the (b, h, n) dimensions of q, k, v and o; the head dim d is contiguous.  Views such as the
 * [B, H, N, D] transpose of a [B, N, H, D] (GPT-style [B, T, H*D]) buffer are read and written in
 * place, without .contiguous() copies.  Each stride must be positive and a multiple of 16 bytes;
 * o must not overlap itself or the inputs. */
typedef struct fa_strides {
  long long q[3];
  long long k[3];
  long long v[3];
  long long o[3];
} fa_strides_t;

/* fa_forward over strided views (see fa_strides_t); lse stays contiguous [B, H, N].  Same
 * return codes as fa_forward; bad strides are cudaErrorInvalidValue. */
int fa_forward_strided(int impl, int dtype, const void* q, const void* k, const void* v, void* o,
                       float* lse, void* workspace, const fa_params_t* p, const fa_strides_t* st,
                       cudaStream_t stream);

/* No counterpart in the reference, whose roadmap lists split-KV decoding with an LSE-weighted
 * combine (the reason the forward returns LSE, attention.cuh:39-40).  Merges n_splits partial
 * results of the same queries over disjoint key sets -- e.g. the steps of ring / context-parallel
 * attention, or KV chunks computed separately:
 *   lse = ln sum_i exp(lse_i),  o = sum_i exp(lse_i - lse) * o_i.
 * o_parts / lse_parts are HOST arrays of n_splits device pointers to contiguous [B, H, N, D]
 * partials of `dtype` (16-byte aligned) and [B, H, N] fp32 natural-log LSEs; a partial row with
 * lse = +inf or -inf saw no key and gets weight 0; a row with no keys anywhere gets o = 0,
 * lse = +inf (the forward's convention, softmax_math.cuh:64-68).  Writes contiguous o and lse,
 * which must not alias the partials.  D is 64 or 128; 1 <= n_splits <= FA_COMBINE_MAX_SPLITS. */
#define FA_COMBINE_MAX_SPLITS 64
int fa_combine(int dtype, int n_splits, const void* const* o_parts, const float* const* lse_parts,
               void* o, float* lse, int B, int H, int N, int D, cudaStream_t stream);

/* No counterpart in the reference: fa_forward with no workspace argument and no allocation, for
 * callers that cannot allocate device memory at call time -- a plugin inside a runtime that
 * reserves all device memory up front and gives it no allocator -- and for loops that avoid
 * cudaMalloc/cudaFree because those can synchronize the device.  Paths that need scratch (fp32 on
 * FA_IMPL_FUSED: fa_workspace_bytes > 0) use a fixed device array of FA_NOALLOC_SCRATCH_BYTES
 * (64 MiB per CUDA context that uses it, held until the process exits); a problem needing more
 * (e.g. B=8 H=16 N=4096 D=128 fp32, 768 MiB) returns cudaErrorInvalidValue without launching
 * anything.  B=2 H=8 N=2048 D=128 fp32 needs 48 MiB.  Invalid or unsupported arguments return the
 * same codes as fa_forward.  The array is shared by all calls in a context and keeps the last
 * call's contents, so calls whose executions overlap on the GPU (other streams or host threads)
 * race on it.  Its address is looked up on each call in the caller's current context; under
 * CUDA's default lazy module loading the first such call in a context loads the library's module
 * and so allocates the array once: make that first fp32 call (a tiny one will do) before
 * reserving the rest of device memory and before any stream capture.  fp16/bf16 need no scratch
 * and run exactly as fa_forward. */
#define FA_NOALLOC_SCRATCH_BYTES (64u * 1024u * 1024u)
int fa_forward_noalloc(int impl, int dtype, const void* q, const void* k, const void* v, void* o,
                       float* lse, const fa_params_t* p, cudaStream_t stream);
/* Size of that scratch array in bytes (FA_NOALLOC_SCRATCH_BYTES). */
size_t fa_noalloc_scratch_bytes(void);

/* fa::workspace_bytes (attention.cuh:51; src/dispatch.cu:163-168).  0 for fp16/bf16.  For fp32
 * (FA_IMPL_FUSED, tf32 tensor cores) 4*D*N*(B*H + 2*B*Hkv) bytes: q, k and v rounded to tf32
 * (round to nearest) before the kernel reads them, instead of the tensor core's truncation. */
size_t fa_workspace_bytes(int impl, int dtype, const fa_params_t* p);

/* fa::impl_supports (attention.cuh:56; src/dispatch.cu:170-175).  `sm` = major*10+minor. */
int fa_impl_supports(int impl, int dtype, int D, int sm);

/* fa::set_debug_overrides / get_debug_overrides (attention.cuh:60-66; src/dispatch.cu:177-189).
 * block_m: 0 or 128 (query rows per tile); block_n: 0, 32, 64 or 128 (keys per tile).
 * Other values make fa_forward return cudaErrorInvalidValue, like the reference's
 * non-instantiated variants (src/stage5_tuned.cu:934-950).  With from_env != 0 the
 * FA_FORCE_BR / FA_FORCE_BC environment variables override the stored values. */
void fa_set_debug_overrides(int block_m, int block_n);
void fa_get_debug_overrides(int from_env, int* block_m, int* block_n);

/* fa::impl_name / dtype_name / dtype_size (attention.cuh:67-69; src/dispatch.cu:191-230). */
const char* fa_impl_name(int impl);
const char* fa_dtype_name(int dtype);
size_t fa_dtype_size(int dtype);

/* No counterpart in the reference (its kernels never wait on anything).  Every mbarrier wait
 * in the sm_100a kernel is bounded; a wait that runs out records a cause bit in a device-side
 * status word, the kernel drains its own copies, frees its tensor memory and exits normally.
 * This call synchronises the current device, returns cudaErrorLaunchTimeout (702) if any
 * launch since the previous call timed out (cudaErrorAssert (710) instead when a build made
 * with -DFA_DEBUG_CHECKS found an index out of range; else the device's sticky error, or
 * cudaSuccess),
 * stores the cause bits in *detail when detail != NULL, and clears the status word. */
int fa_last_device_error(unsigned int* detail);

/* No counterpart in the reference: the time limit of each device-side wait, in nanoseconds
 * (default 2e9).  Used by the failure-detection tests to make an injected stall end quickly. */
void fa_set_wait_timeout_ns(unsigned long long ns);

/* No counterpart in the reference: test-only fault injection on the host side of the launch.
 * When tile >= 0, the producer warp of every CTA skips the K load of key tile `tile`, so the
 * MMA warp's bounded wait for it runs out (no GPU fault, no trap).  -1 disables. */
void fa_debug_set_skip_kv_tile(int tile);

#ifdef __cplusplus
}
#endif

#endif /* FA_SM100_H_ */
