// dispatch.cu -- the C ABI declared in include/fa_sm100.h.
//
// Reference counterpart: src/dispatch.cu (the fa::forward registry, contract gate, validation
// and FA_FORCE_BR/BC overrides).  This build has exactly one implementation -- the sm_100a
// tcgen05 kernel in fa_fwd_sm100.cu, registered as Impl::Tuned (fp16/bf16) and Impl::Fused
// (fp32 on tf32, and fp16) -- so the registry collapses to a single gate; there is no fallback
// and no other backend.  Validation order, error codes and the
// FA_VERBOSE convention follow the reference (src/dispatch.cu:96-161,
// src/stage5_tuned.cu:977-1037).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "fa_launch.h"
#include "fa_sm100.h"

namespace {

bool verbose() {
  static const bool v = std::getenv("FA_VERBOSE") != nullptr;
  return v;
}

// Positive integer from the environment; 0 when unset/empty/malformed (malformed is reported
// once so a typo cannot silently test nothing) -- src/dispatch.cu:118-131.
int env_positive_int(const char* name) {
  const char* s = std::getenv(name);
  if (s == nullptr || *s == '\0') return 0;
  char* end = nullptr;
  const long v = std::strtol(s, &end, 10);
  if (end == s || *end != '\0' || v <= 0 || v > (1 << 20)) {
    std::fprintf(stderr, "fa: ignoring %s='%s' (expected a positive integer)\n", name, s);
    return 0;
  }
  return static_cast<int>(v);
}

int g_block_m = 0;  // set_debug_overrides state (process-global, not thread-safe)
int g_block_n = 0;
unsigned long long g_timeout_ns = 2000000000ull;
int g_skip_kv_tile = -1;

bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

// nullptr when valid, else the reason (printed only under FA_VERBOSE).
const char* validate(int dtype, const void* q, const void* k, const void* v, const void* o,
                     const float* lse, const fa_params_t* p) {
  if (p == nullptr) return "params must be non-null";
  if (p->B <= 0 || p->H <= 0 || p->Hkv <= 0 || p->N <= 0 || p->D <= 0)
    return "B,H,Hkv,N,D must be > 0";
  if (p->D != 64 && p->D != 128) return "D must be 64 or 128";
  if (p->N % 32 != 0) return "N % 32 != 0 (ragged N is a documented in-window limitation)";
  if (p->H % p->Hkv != 0) return "H % Hkv != 0";
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr)
    return "q/k/v/o must be non-null";
  if (fa_dtype_size(dtype) == 0) return "unknown dtype";
  if (lse == nullptr) return "lse must be non-null";
  if (!(p->scale > 0.0f) || !std::isfinite(p->scale)) return "scale must be finite and > 0";
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return "q/k/v/o must be 16-byte aligned";
  if ((p->N + 127) / 128 > 65535) return "N too large (more than 65535 query tiles)";
  return nullptr;
}

cudaError_t current_sm(int* sm) {
  int dev = 0, major = 0, minor = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
    return e;
  if ((e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
    return e;
  *sm = major * 10 + minor;
  return cudaSuccess;
}

}  // namespace

extern "C" {

size_t fa_dtype_size(int dtype) {
  switch (dtype) {
    case FA_DTYPE_F32:
      return 4;
    case FA_DTYPE_F16:
    case FA_DTYPE_BF16:
      return 2;
    default:
      return 0;
  }
}

const char* fa_dtype_name(int dtype) {
  switch (dtype) {
    case FA_DTYPE_F32:
      return "fp32";
    case FA_DTYPE_F16:
      return "fp16";
    case FA_DTYPE_BF16:
      return "bf16";
    default:
      return "unknown";
  }
}

const char* fa_impl_name(int impl) {
  switch (impl) {
    case FA_IMPL_NAIVE:
      return "naive";
    case FA_IMPL_TILED:
      return "tiled";
    case FA_IMPL_FUSED:
      return "fused";
    case FA_IMPL_WMMA:
      return "wmma";
    case FA_IMPL_TUNED:
      return "tuned";
    default:
      return "unknown";
  }
}

// The kernel is compiled for sm_100a only (the 'a' target runs on compute capability 10.0).
// Support matrix per stage as in the reference (src/dispatch.cu:76-89): Tuned takes fp16/bf16,
// Fused takes fp32/fp16.  Both run the one tcgen05 kernel (fp32 on the tf32 tensor-core path);
// the naive/tiled/wmma teaching stages are not built.
int fa_impl_supports(int impl, int dtype, int D, int sm) {
  if (D != 64 && D != 128) return 0;
  if (sm != 100) return 0;
  switch (impl) {
    case FA_IMPL_TUNED:
      if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return 0;
      break;
    case FA_IMPL_FUSED:
      if (dtype != FA_DTYPE_F32 && dtype != FA_DTYPE_F16) return 0;
      break;
    default:
      return 0;
  }
  return fa_sm100::block_n_supported(dtype, D, fa_sm100::default_block_n(dtype, D, 0, 0)) ? 1 : 0;
}

// 0 for fp16/bf16.  fp32 (Impl::Fused) stages tf32-rounded copies of q, k, v in the workspace.
size_t fa_workspace_bytes(int impl, int dtype, const fa_params_t* p) {
  if (p == nullptr || impl != FA_IMPL_FUSED || dtype != FA_DTYPE_F32) return 0;
  if (p->B <= 0 || p->H <= 0 || p->Hkv <= 0 || p->N <= 0 || p->D <= 0) return 0;
  return fa_sm100::workspace_bytes_f32(p->B, p->H, p->Hkv, p->N, p->D);
}

void fa_set_debug_overrides(int block_m, int block_n) {
  g_block_m = block_m;
  g_block_n = block_n;
}

void fa_get_debug_overrides(int from_env, int* block_m, int* block_n) {
  int bm = g_block_m, bn = g_block_n;
  if (from_env) {
    if (const int e = env_positive_int("FA_FORCE_BR")) bm = e;
    if (const int e = env_positive_int("FA_FORCE_BC")) bn = e;
  }
  if (block_m) *block_m = bm;
  if (block_n) *block_n = bn;
}

void fa_set_wait_timeout_ns(unsigned long long ns) { g_timeout_ns = ns > 0 ? ns : 1; }

void fa_debug_set_skip_kv_tile(int tile) { g_skip_kv_tile = tile < 0 ? -1 : tile; }

int fa_last_device_error(unsigned int* detail) {
  return static_cast<int>(fa_sm100::read_and_clear_status(detail));
}

}  // extern "C"

namespace {

// Stride rules of a strided view: positive element strides whose byte sizes are multiples of 16
// (the TMA tensor-map rule; with a 16-byte-aligned base every row then starts 16-byte aligned).
const char* check_strides(const long long st[3], size_t eb, const char* name) {
  for (int i = 0; i < 3; ++i) {
    if (st[i] <= 0) return name;
    if ((static_cast<unsigned long long>(st[i]) * eb) % 16 != 0) return name;
    if (static_cast<unsigned long long>(st[i]) * eb >= (1ull << 40)) return name;
  }
  return nullptr;
}

}  // namespace

namespace fa_sm100 {

// Every check fa_forward makes before it launches, in its order and with its error codes:
// parameters, strides (when given), the implementation on the current device, the workspace.
cudaError_t check_forward_args(int impl, int dtype, const void* q, const void* k, const void* v,
                               const void* o, const float* lse, const void* workspace,
                               bool need_workspace, const fa_params_t* p, const fa_strides_t* st) {
  if (const char* why = validate(dtype, q, k, v, o, lse, p)) {
    if (verbose()) std::fprintf(stderr, "fa_forward: invalid params: %s\n", why);
    return cudaErrorInvalidValue;
  }
  if (st != nullptr) {
    const size_t eb = fa_dtype_size(dtype);
    const char* bad = check_strides(st->q, eb, "q");
    if (bad == nullptr) bad = check_strides(st->k, eb, "k");
    if (bad == nullptr) bad = check_strides(st->v, eb, "v");
    if (bad == nullptr) bad = check_strides(st->o, eb, "o");
    if (bad != nullptr) {
      if (verbose()) {
        std::fprintf(stderr, "fa_forward_strided: %s strides must be positive multiples of 16 "
                             "bytes\n", bad);
      }
      return cudaErrorInvalidValue;
    }
  }
  int sm = 0;
  if (const cudaError_t e = current_sm(&sm)) return e;
  if (!fa_impl_supports(impl, dtype, p->D, sm)) {
    if (verbose()) {
      std::fprintf(stderr, "fa_forward: %s/%s/D=%d not supported on sm_%d in this build\n",
                   fa_impl_name(impl), fa_dtype_name(dtype), p->D, sm);
    }
    return cudaErrorNotSupported;
  }
  if (need_workspace && fa_workspace_bytes(impl, dtype, p) > 0 &&
      (workspace == nullptr || !aligned16(workspace))) {
    if (verbose()) {
      std::fprintf(stderr, "fa_forward: workspace must be non-null and 16-byte aligned "
                           "(fa_workspace_bytes > 0)\n");
    }
    return cudaErrorInvalidValue;
  }
  return cudaSuccess;
}

}  // namespace fa_sm100

namespace {

int forward_impl(int impl, int dtype, const void* q, const void* k, const void* v, void* o,
                 float* lse, void* workspace, const fa_params_t* p, const fa_strides_t* st,
                 cudaStream_t stream) {
  if (const cudaError_t e =
          fa_sm100::check_forward_args(impl, dtype, q, k, v, o, lse, workspace, true, p, st)) {
    return static_cast<int>(e);
  }
  int bm = 0, bn = 0;
  fa_get_debug_overrides(1, &bm, &bn);
  if (bm != 0 && bm != 128) {
    if (verbose()) std::fprintf(stderr, "fa_forward: block_m=%d is not built (0 or 128)\n", bm);
    return cudaErrorInvalidValue;
  }
  if (bn == 0) bn = fa_sm100::default_block_n(dtype, p->D, p->N, p->causal);
  if (!fa_sm100::block_n_supported(dtype, p->D, bn)) {
    if (verbose()) {
      std::fprintf(stderr, "fa_forward: block_n=%d is not built (0, 32, 64 or 128)\n", bn);
    }
    return cudaErrorInvalidValue;
  }
  fa_sm100::LaunchArgs a;
  a.dtype = dtype;
  a.q = q;
  a.k = k;
  a.v = v;
  a.o = o;
  a.lse = lse;
  a.B = p->B;
  a.H = p->H;
  a.Hkv = p->Hkv;
  a.N = p->N;
  a.D = p->D;
  a.scale = p->scale;
  a.causal = p->causal != 0;
  a.block_n = bn;
  a.timeout_ns = g_timeout_ns;
  a.skip_kv_tile = g_skip_kv_tile;
  a.workspace = workspace;
  if (st != nullptr) {
    for (int i = 0; i < 3; ++i) {
      a.sq[i] = st->q[i];
      a.sk[i] = st->k[i];
      a.sv[i] = st->v[i];
      a.so[i] = st->o[i];
    }
  } else {
    // Contiguous [B, H, N, D] (q, o) and [B, Hkv, N, D] (k, v).
    const long long nd = static_cast<long long>(p->N) * p->D;
    const long long cq[3] = {static_cast<long long>(p->H) * nd, nd, p->D};
    const long long ckv[3] = {static_cast<long long>(p->Hkv) * nd, nd, p->D};
    for (int i = 0; i < 3; ++i) {
      a.sq[i] = cq[i];
      a.so[i] = cq[i];
      a.sk[i] = ckv[i];
      a.sv[i] = ckv[i];
    }
  }
  return static_cast<int>(fa_sm100::launch_forward(a, stream));
}

}  // namespace

extern "C" {

int fa_forward(int impl, int dtype, const void* q, const void* k, const void* v, void* o,
               float* lse, void* workspace, const fa_params_t* p, cudaStream_t stream) {
  return forward_impl(impl, dtype, q, k, v, o, lse, workspace, p, nullptr, stream);
}

int fa_forward_strided(int impl, int dtype, const void* q, const void* k, const void* v, void* o,
                       float* lse, void* workspace, const fa_params_t* p, const fa_strides_t* st,
                       cudaStream_t stream) {
  if (st == nullptr) return cudaErrorInvalidValue;
  return forward_impl(impl, dtype, q, k, v, o, lse, workspace, p, st, stream);
}

}  // extern "C"
