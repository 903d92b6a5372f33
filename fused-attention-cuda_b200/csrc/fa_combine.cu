// fa_combine.cu -- LSE-weighted merge of attention partials over disjoint key sets (split-KV /
// ring attention), the combine step the reference lists on its roadmap next to the LSE output
// (include/fa/attention.cuh:39-40; include/fa/softmax_math.cuh:66-68 fixes the sentinels).
//
// For each query row with partials (O_i, lse_i), lse_i in natural-log units:
//   lse = ln sum_i exp(lse_i),  O = sum_i exp(lse_i - lse) * O_i,
// computed as m = max_i lse_i, w_i = exp(lse_i - m), l = sum_i w_i, lse = m + ln l.  A partial
// whose rows saw no key reports lse_i = +inf (the forward's non-split convention) or -inf; both
// mean "no keys" and get weight 0.  A row with no keys in any partial gets O = 0, lse = +inf, like
// the forward.  Accumulation is fp32; O is rounded to the output type once.
//
// HBM-bound: per row it reads n_splits * (D * elem + 4) bytes and writes D * elem + 4.  One thread
// per 16-byte chunk of a row (D * elem / 16 threads per row), a grid-stride loop over rows.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <type_traits>

#include "fa_sm100.h"

namespace {

constexpr int kMaxSplits = FA_COMBINE_MAX_SPLITS;

struct CombineArgs {
  const void* o_parts[kMaxSplits];
  const float* lse_parts[kMaxSplits];
  int n_splits;
  long long rows;  // B * H * N
  void* o;
  float* lse;
};

__device__ __forceinline__ bool no_keys(float x) { return !(fabsf(x) < INFINITY); }

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]);
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&f)[8]);
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float (&f)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// T = fp16/bf16: 8 elements per 16-byte chunk; T = float: 4 (stored as the first half of f).
template <typename T, int D>
__global__ void __launch_bounds__(256) fa_combine_kernel(const CombineArgs a) {
  constexpr int kElems = std::is_same<T, float>::value ? 4 : 8;  // per 16-byte chunk
  constexpr int kChunks = D / kElems;                               // threads per row
  const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long t = tid; t < a.rows * kChunks; t += stride) {
    const long long row = t / kChunks;
    const int c = static_cast<int>(t - row * kChunks);
    float m = -INFINITY;
    for (int i = 0; i < a.n_splits; ++i) {
      const float x = a.lse_parts[i][row];
      if (!no_keys(x)) m = fmaxf(m, x);
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float l = 0.f;
    if (m != -INFINITY) {
      for (int i = 0; i < a.n_splits; ++i) {
        const float x = a.lse_parts[i][row];
        if (no_keys(x)) continue;
        const float wgt = expf(x - m);
        l += wgt;
        const T* src = static_cast<const T*>(a.o_parts[i]) + row * D + c * kElems;
        float f[8];
        if constexpr (std::is_same<T, float>::value) {
          const float4 u = *reinterpret_cast<const float4*>(src);
          f[0] = u.x;
          f[1] = u.y;
          f[2] = u.z;
          f[3] = u.w;
        } else {
          load8<T>(src, f);
        }
#pragma unroll
        for (int e = 0; e < kElems; ++e) acc[e] = fmaf(wgt, f[e], acc[e]);
      }
    }
    const float inv_l = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int e = 0; e < kElems; ++e) acc[e] *= inv_l;
    T* dst = static_cast<T*>(a.o) + row * D + c * kElems;
    if constexpr (std::is_same<T, float>::value) {
      *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    } else {
      store8<T>(dst, acc);
    }
    if (c == 0) a.lse[row] = l > 0.f ? m + logf(l) : INFINITY;
  }
}

template <typename T>
cudaError_t launch(const CombineArgs& a, int D, cudaStream_t s) {
  int dev = 0, sms = 148;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
  const int per_row = D * static_cast<int>(sizeof(T)) / 16;
  const long long threads = a.rows * per_row;
  long long blocks = (threads + 255) / 256;
  const long long cap = static_cast<long long>(sms) * 16;
  if (blocks > cap) blocks = cap;
  if (D == 64) {
    fa_combine_kernel<T, 64><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a);
  } else {
    fa_combine_kernel<T, 128><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a);
  }
  return cudaGetLastError();
}

bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int fa_combine(int dtype, int n_splits, const void* const* o_parts,
                          const float* const* lse_parts, void* o, float* lse, int B, int H, int N,
                          int D, cudaStream_t stream) {
  if (n_splits < 1 || n_splits > kMaxSplits) return cudaErrorInvalidValue;
  if (B <= 0 || H <= 0 || N <= 0 || (D != 64 && D != 128)) return cudaErrorInvalidValue;
  if (o_parts == nullptr || lse_parts == nullptr || o == nullptr || lse == nullptr) {
    return cudaErrorInvalidValue;
  }
  if (fa_dtype_size(dtype) == 0) return cudaErrorInvalidValue;
  CombineArgs a;
  for (int i = 0; i < n_splits; ++i) {
    if (o_parts[i] == nullptr || lse_parts[i] == nullptr || !aligned16(o_parts[i])) {
      return cudaErrorInvalidValue;
    }
    a.o_parts[i] = o_parts[i];
    a.lse_parts[i] = lse_parts[i];
  }
  if (!aligned16(o)) return cudaErrorInvalidValue;
  a.n_splits = n_splits;
  a.rows = static_cast<long long>(B) * H * N;
  a.o = o;
  a.lse = lse;
  switch (dtype) {
    case FA_DTYPE_F16:
      return static_cast<int>(launch<__half>(a, D, stream));
    case FA_DTYPE_BF16:
      return static_cast<int>(launch<__nv_bfloat16>(a, D, stream));
    case FA_DTYPE_F32:
      return static_cast<int>(launch<float>(a, D, stream));
    default:
      return cudaErrorInvalidValue;
  }
}
