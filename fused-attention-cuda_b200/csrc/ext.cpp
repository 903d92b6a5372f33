// fused_attn._C -- PyTorch operator surface over the C ABI in include/fa_sm100.h.
//
// Reference counterpart: python/fused_attn/ext.cpp.  Same library name (fused_attn), same
// validation messages (make_params, ext.cpp:82-126), same bare PyInit__C module (ext.cpp:240-253)
// so `from . import _C` runs the TORCH_LIBRARY initialisers.  One deliberate change:
//   fused_attn::forward(Tensor q, Tensor k, Tensor v, bool is_causal, float scale)
//       -> (Tensor, Tensor)                           (O, LSE) -- the reference returns O only
// because the B200 build's contract is "forward -> (O, LSE)".  forward_stage keeps its
// (Tensor, Tensor) schema; its LSE is empty for the stages that do not write one (1, 2).
//
// Host C++ only: every launch happens behind fa_forward() in libfa_sm100.so.
#include <Python.h>  // first, per the CPython docs
// (blank comment line keeps include sorters from moving Python.h)

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/library.h>

#include <cmath>
#include <cstdint>
#include <limits>
#include <string>
#include <tuple>
#include <vector>

#include "fa_sm100.h"

namespace {

// The reference's stage numbering (fa::Impl): 1..5, with an LSE from stage 3 up.  Constructing a
// Stage is the range check.
struct Stage {
  static constexpr int kLowest = 1;
  static constexpr int kHighest = 5;
  static constexpr int kFirstWithLse = 3;
  int value;
  explicit Stage(int64_t s) : value(static_cast<int>(s)) {
    TORCH_CHECK(s >= kLowest && s <= kHighest, "fused_attn: stage must be in 1..5, got ", s);
  }
  bool writes_lse() const { return value >= kFirstWithLse; }
};

int to_fa_dtype(at::ScalarType t) {
  if (t == at::kFloat) return FA_DTYPE_F32;
  if (t == at::kHalf) return FA_DTYPE_F16;
  TORCH_CHECK(t == at::kBFloat16, "fused_attn: unsupported dtype ", t,
              " (supported: float32, float16, bfloat16)");
  return FA_DTYPE_BF16;
}

int dtype_from_name(const std::string& name) {
  if (name == "fp32") return FA_DTYPE_F32;
  if (name == "fp16") return FA_DTYPE_F16;
  TORCH_CHECK(name == "bf16", "fused_attn: unknown dtype name '", name,
              "' (expected fp32, fp16 or bf16)");
  return FA_DTYPE_BF16;
}

// fa_impl_supports' `sm` (major * 10 + minor) for a CUDA device index (-1: the current one).
int sm_number(int device_index = -1) {
  const cudaDeviceProp* prop = device_index < 0 ? at::cuda::getCurrentDeviceProperties()
                                                : at::cuda::getDeviceProperties(device_index);
  return 10 * prop->major + prop->minor;
}

// A size or knob narrowed to the C ABI's `int` fields, rejected when it does not fit.
int abi_int(int64_t v, const char* what) {
  const bool fits = v >= 0 && v <= static_cast<int64_t>(std::numeric_limits<int>::max());
  TORCH_CHECK(fits, "fused_attn: ", what, "=", v, " does not fit fa_params_t (int)");
  return static_cast<int>(v);
}

// Input contract (reference ext.cpp:82-126): every violation is a RuntimeError, never a fault.
// With `strided`, q/k/v may be any [B, H, N, D] views whose head dim is contiguous and whose other
// strides are positive multiples of 16 bytes (no counterpart in the reference, which requires
// contiguous inputs).
fa_params_t make_params(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                        bool is_causal, double scale, bool strided = false) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(),
              "fused_attn: q, k, v must be CUDA tensors");
  TORCH_CHECK(q.device() == k.device() && q.device() == v.device(),
              "fused_attn: q, k, v must live on the same device");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4,
              "fused_attn: q, k, v must be [B, H, N, D]; got ", q.dim(), "-D, ", k.dim(), "-D, ",
              v.dim(), "-D");
  if (!strided) {
    TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(),
                "fused_attn: q, k, v must be contiguous [B, H, N, D] (call .contiguous())");
  } else {
    for (const at::Tensor* t : {&q, &k, &v}) {
      TORCH_CHECK(t->dim() == 4 && t->stride(3) == 1,
                  "fused_attn: strided views need a contiguous head dim (stride(3) == 1)");
      for (int d = 0; d < 3; ++d) {
        TORCH_CHECK(t->stride(d) > 0 && (t->stride(d) * t->element_size()) % 16 == 0,
                    "fused_attn: strided views need positive strides that are multiples of 16 "
                    "bytes; got stride(", d, ") = ", t->stride(d));
      }
    }
  }
  for (const at::Tensor* t : {&q, &k, &v}) {
    TORCH_CHECK(reinterpret_cast<std::uintptr_t>(t->data_ptr()) % 16 == 0,
                "fused_attn: q/k/v must be 16-byte aligned (use a fresh contiguous tensor)");
  }
  TORCH_CHECK(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(),
              "fused_attn: q, k, v must share one dtype; got ", q.scalar_type(), ", ",
              k.scalar_type(), ", ", v.scalar_type());
  (void)to_fa_dtype(q.scalar_type());

  const int64_t B = q.size(0), H = q.size(1), N = q.size(2), D = q.size(3);
  const int64_t Hkv = k.size(1);
  TORCH_CHECK(k.size(0) == B && v.size(0) == B, "fused_attn: batch mismatch between q, k, v");
  TORCH_CHECK(v.size(1) == Hkv, "fused_attn: k and v must have the same number of heads");
  TORCH_CHECK(k.size(2) == N && v.size(2) == N,
              "fused_attn: Nq == Nkv is required in-window (got Nq=", N, ", Nkv=", k.size(2), ")");
  TORCH_CHECK(k.size(3) == D && v.size(3) == D, "fused_attn: head-dim mismatch between q, k, v");
  TORCH_CHECK(D == 64 || D == 128, "fused_attn: D must be 64 or 128, got ", D);
  TORCH_CHECK(N % 32 == 0, "fused_attn: N must be a multiple of 32, got ", N,
              " (ragged sequence lengths are a stated in-window limitation)");
  TORCH_CHECK(Hkv >= 1 && H % Hkv == 0, "fused_attn: H=", H, " must be a multiple of Hkv=", Hkv);
  TORCH_CHECK(scale > 0.0 && std::isfinite(scale), "fused_attn: scale must be finite and > 0, got ",
              scale);

  fa_params_t p;
  p.B = abi_int(B, "B");
  p.H = abi_int(H, "H");
  p.Hkv = abi_int(Hkv, "Hkv");
  p.N = abi_int(N, "N");
  p.D = abi_int(D, "D");
  p.scale = static_cast<float>(scale);
  p.causal = is_causal ? 1 : 0;
  return p;
}

// The stage's outputs and scratch on q's device.  O takes q's layout (empty_like keeps the strides
// of a dense view, e.g. the [B, H, N, D] transpose of a [B, N, H, D] buffer), so a head merge after
// the op is a free view too.  The LSE is [B, H, N] fp32, or empty for a stage that writes none.
struct StageBuffers {
  at::Tensor o, lse, workspace;
  StageBuffers(const at::Tensor& q, const fa_params_t& p, Stage stage, int dtype) {
    const auto f32 = q.options().dtype(at::kFloat);
    o = at::empty_like(q);
    lse = stage.writes_lse() ? at::empty({p.B, p.H, p.N}, f32) : at::empty({0}, f32);
    const std::size_t scratch = fa_workspace_bytes(stage.value, dtype, &p);
    if (scratch > 0) {
      workspace = at::empty({static_cast<int64_t>(scratch)}, q.options().dtype(at::kByte));
    }
  }
  float* lse_ptr() { return lse.numel() > 0 ? lse.data_ptr<float>() : nullptr; }
  void* workspace_ptr() { return workspace.defined() ? workspace.data_ptr() : nullptr; }
};

std::tuple<at::Tensor, at::Tensor> run_stage(const at::Tensor& q, const at::Tensor& k,
                                             const at::Tensor& v, bool is_causal, double scale,
                                             Stage stage, bool strided = false) {
  const fa_params_t p = make_params(q, k, v, is_causal, scale, strided);
  const c10::cuda::CUDAGuard guard(q.device());
  const int impl = stage.value;
  const int dtype = to_fa_dtype(q.scalar_type());
  const int sm = sm_number(q.device().index());
  TORCH_CHECK(fa_impl_supports(impl, dtype, p.D, sm), "fused_attn: stage ", impl, " (",
              fa_impl_name(impl), ") is not implemented for ", fa_dtype_name(dtype), " D=", p.D,
              " on sm_", sm);
  StageBuffers out(q, p, stage, dtype);
  at::Tensor& o = out.o;
  const bool has_lse = stage.writes_lse();
  void* ws_ptr = out.workspace_ptr();
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream(q.device().index()).stream();
  int err;
  if (strided) {
    TORCH_CHECK(o.stride(3) == 1, "fused_attn: output layout has a non-contiguous head dim");
    fa_strides_t st;
    const at::Tensor* ts[4] = {&q, &k, &v, &o};
    long long* dst[4] = {st.q, st.k, st.v, st.o};
    for (int t = 0; t < 4; ++t) {
      for (int d = 0; d < 3; ++d) dst[t][d] = static_cast<long long>(ts[t]->stride(d));
    }
    err = fa_forward_strided(impl, dtype, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                             has_lse ? out.lse_ptr() : nullptr, ws_ptr, &p, &st, stream);
  } else {
    err = fa_forward(impl, dtype, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                     has_lse ? out.lse_ptr() : nullptr, ws_ptr, &p, stream);
  }
  TORCH_CHECK(err == 0, "fused_attn: stage ", impl, " (", fa_impl_name(impl),
              ") failed: ", cudaGetErrorString(static_cast<cudaError_t>(err)));
  return std::make_tuple(std::move(out.o), std::move(out.lse));
}

// The stage `forward` runs: the highest one with an LSE that this device supports for the dtype
// and head dim (the reference's forward picks its best stage the same way, ext.cpp:174-188).
Stage best_stage(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool is_causal,
                 double scale, bool strided) {
  const fa_params_t p = make_params(q, k, v, is_causal, scale, strided);
  const int dtype = to_fa_dtype(q.scalar_type());
  const int sm = sm_number(q.device().index());
  int chosen = 0;
  for (int s = Stage::kHighest; s >= Stage::kFirstWithLse && chosen == 0; --s) {
    if (fa_impl_supports(s, dtype, p.D, sm)) chosen = s;
  }
  TORCH_CHECK(chosen != 0, "fused_attn: no stage is implemented for ", fa_dtype_name(dtype),
              " D=", p.D, " on sm_", sm);
  return Stage(chosen);
}

std::tuple<at::Tensor, at::Tensor> forward_cuda(const at::Tensor& q, const at::Tensor& k,
                                                const at::Tensor& v, bool is_causal,
                                                double scale) {
  return run_stage(q, k, v, is_causal, scale, best_stage(q, k, v, is_causal, scale, false));
}

// forward over strided [B, H, N, D] views (no counterpart in the reference): same stage choice.
std::tuple<at::Tensor, at::Tensor> forward_strided_cuda(const at::Tensor& q, const at::Tensor& k,
                                                        const at::Tensor& v, bool is_causal,
                                                        double scale) {
  return run_stage(q, k, v, is_causal, scale, best_stage(q, k, v, is_causal, scale, true), true);
}

std::tuple<at::Tensor, at::Tensor> forward_stage_cuda(const at::Tensor& q, const at::Tensor& k,
                                                      const at::Tensor& v, bool is_causal,
                                                      double scale, int64_t stage) {
  return run_stage(q, k, v, is_causal, scale, Stage(stage));
}

// LSE-weighted merge of partials over disjoint key sets (no counterpart in the reference).
std::tuple<at::Tensor, at::Tensor> combine_cuda(at::TensorList o_parts, at::TensorList lse_parts) {
  TORCH_CHECK(!o_parts.empty() && o_parts.size() == lse_parts.size(),
              "fused_attn: combine needs as many LSE tensors as O partials (at least one)");
  TORCH_CHECK(o_parts.size() <= FA_COMBINE_MAX_SPLITS, "fused_attn: combine takes at most ",
              FA_COMBINE_MAX_SPLITS, " partials, got ", o_parts.size());
  const at::Tensor& o0 = o_parts[0];
  TORCH_CHECK(o0.is_cuda() && o0.dim() == 4, "fused_attn: partials must be CUDA [B, H, N, D]");
  const int64_t B = o0.size(0), H = o0.size(1), N = o0.size(2), D = o0.size(3);
  TORCH_CHECK(D == 64 || D == 128, "fused_attn: D must be 64 or 128, got ", D);
  std::vector<const void*> op;
  std::vector<const float*> lp;
  for (size_t i = 0; i < o_parts.size(); ++i) {
    const at::Tensor& o = o_parts[i];
    const at::Tensor& l = lse_parts[i];
    TORCH_CHECK(o.device() == o0.device() && l.device() == o0.device(),
                "fused_attn: combine inputs must live on one device");
    TORCH_CHECK(o.sizes() == o0.sizes() && o.scalar_type() == o0.scalar_type() &&
                    o.is_contiguous(),
                "fused_attn: O partials must be contiguous with one shape and dtype");
    TORCH_CHECK(l.scalar_type() == at::kFloat && l.is_contiguous() && l.dim() == 3 &&
                    l.size(0) == B && l.size(1) == H && l.size(2) == N,
                "fused_attn: LSE partials must be contiguous fp32 [B, H, N]");
    TORCH_CHECK(reinterpret_cast<std::uintptr_t>(o.data_ptr()) % 16 == 0,
                "fused_attn: O partials must be 16-byte aligned");
    op.push_back(o.data_ptr());
    lp.push_back(l.data_ptr<float>());
  }
  const c10::cuda::CUDAGuard guard(o0.device());
  at::Tensor out = at::empty_like(o0, at::MemoryFormat::Contiguous);
  at::Tensor lse = at::empty({B, H, N}, o0.options().dtype(at::kFloat));
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream(o0.device().index()).stream();
  const int err = fa_combine(to_fa_dtype(o0.scalar_type()), static_cast<int>(op.size()), op.data(),
                             lp.data(), out.data_ptr(), lse.data_ptr<float>(),
                             abi_int(B, "B"), abi_int(H, "H"), abi_int(N, "N"),
                             abi_int(D, "D"), stream);
  TORCH_CHECK(err == 0, "fused_attn: combine failed: ",
              cudaGetErrorString(static_cast<cudaError_t>(err)));
  return std::make_tuple(std::move(out), std::move(lse));
}

void set_debug_overrides_op(int64_t block_m, int64_t block_n) {
  fa_set_debug_overrides(abi_int(block_m, "block_m"), abi_int(block_n, "block_n"));
}

bool impl_supports_op(int64_t stage, std::string dtype, int64_t D) {
  const Stage st(stage);
  if (c10::cuda::device_count() == 0) return false;
  return fa_impl_supports(st.value, dtype_from_name(dtype), abi_int(D, "D"), sm_number()) != 0;
}

std::string impl_name_op(int64_t stage) { return fa_impl_name(Stage(stage).value); }

}  // namespace

TORCH_LIBRARY(fused_attn, m) {
  m.def("forward(Tensor q, Tensor k, Tensor v, bool is_causal, float scale) -> (Tensor, Tensor)");
  m.def(
      "forward_strided(Tensor q, Tensor k, Tensor v, bool is_causal, float scale)"
      " -> (Tensor, Tensor)");
  m.def(
      "forward_stage(Tensor q, Tensor k, Tensor v, bool is_causal, float scale, int stage)"
      " -> (Tensor, Tensor)");
  m.def("combine(Tensor[] o_parts, Tensor[] lse_parts) -> (Tensor, Tensor)");
  m.def("set_debug_overrides(int block_m, int block_n) -> ()", &set_debug_overrides_op);
  m.def("impl_supports(int stage, str dtype, int D) -> bool", &impl_supports_op);
  m.def("impl_name(int stage) -> str", &impl_name_op);
}

TORCH_LIBRARY_IMPL(fused_attn, CUDA, m) {
  m.impl("forward", &forward_cuda);
  m.impl("forward_strided", &forward_strided_cuda);
  m.impl("combine", &combine_cuda);
  m.impl("forward_stage", &forward_stage_cuda);
}

// A module with no functions of its own: importing it runs the TORCH_LIBRARY registrations above,
// and the ops are reached as torch.ops.fused_attn.*.
static PyModuleDef g_module = {PyModuleDef_HEAD_INIT, "_C",
                               "B200 SDPA forward; ops under torch.ops.fused_attn", -1};

extern "C" PyObject* PyInit__C(void) { return PyModule_Create(&g_module); }
