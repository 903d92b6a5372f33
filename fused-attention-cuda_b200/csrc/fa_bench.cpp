// fa_bench.cpp -- torch-free benchmark of the SDPA forward through the C ABI alone.
//
// Reference counterpart: bench/bench_main.cu (the reference's fa_bench): seeded inputs, a pre-flight
// launch, an fp64 self-check that must pass before any timing row is written (:589-656, :763),
// then a timed loop with one CUDA-event pair per launch and an L2 flush before each (:517-565).
// This program links libfa_sm100.so through include/fa_sm100.h only -- no PyTorch -- so it is also
// the proof that a non-Python caller can drive the library: everything it needs is a device
// pointer, an fa_params_t and a stream.
//
//   fa_bench [--cfg B2_H8_N2048_D128] [--dtype fp16|bf16] [--causal 0|1] [--seed 2]
//            [--iters 100] [--warmup 10] [--oracle PATH] [--threads T]
//
// Inputs: iid N(0, 1) from a seeded splitmix64 stream (Box-Muller), rounded to the kernel dtype on
// the host.  Self-check: heads (0, 0) and (B-1, H-1) in full against the fp64 CPU oracle
// (oracle/libfa_oracle.so, loaded with dlopen; it is the checker, never the thing timed), fed the
// same rounded inputs upcast to double.  Gates: fp16 O <= 2e-3 and LSE <= 1e-3, bf16 O <= 8e-3 and
// LSE <= 1e-3.  A failed check prints the errors and exits with status 2 without a timing row.
// Output: one JSON line.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "fa_sm100.h"

namespace {

// The oracle's shape record (oracle/fa_oracle.c): same field order and types.
struct OracleShape {
  int B, H, Hkv, N, D;
  double scale;
  int causal;
};
using OracleAttentionFn = int (*)(const double*, const double*, const double*, const OracleShape*,
                                  double*, double*, int);

struct Options {
  int B = 2, H = 8, N = 2048, D = 128;
  int dtype = FA_DTYPE_F16;
  int causal = 1;
  unsigned long long seed = 2;
  int iters = 100, warmup = 10;
  int threads = 0;
  double perturb_oracle = 0.0;  // test hook: added to the oracle's O before the comparison
  std::string oracle;
};

bool check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "fa_bench: %s: %s\n", what, cudaGetErrorString(e));
    return false;
  }
  return true;
}

bool parse(int argc, char** argv, Options* o) {
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    const char* val = i + 1 < argc ? argv[i + 1] : nullptr;
    auto need = [&]() {
      if (val == nullptr) {
        std::fprintf(stderr, "fa_bench: %s needs a value\n", a.c_str());
        std::exit(1);
      }
      ++i;
      return std::string(val);
    };
    if (a == "--cfg") {
      const std::string v = need();
      if (std::sscanf(v.c_str(), "B%d_H%d_N%d_D%d", &o->B, &o->H, &o->N, &o->D) != 4) return false;
    } else if (a == "--dtype") {
      const std::string v = need();
      if (v == "fp16") {
        o->dtype = FA_DTYPE_F16;
      } else if (v == "bf16") {
        o->dtype = FA_DTYPE_BF16;
      } else {
        return false;
      }
    } else if (a == "--causal") {
      o->causal = std::atoi(need().c_str()) != 0;
    } else if (a == "--seed") {
      o->seed = std::strtoull(need().c_str(), nullptr, 10);
    } else if (a == "--iters") {
      o->iters = std::max(1, std::atoi(need().c_str()));
    } else if (a == "--warmup") {
      o->warmup = std::max(0, std::atoi(need().c_str()));
    } else if (a == "--threads") {
      o->threads = std::max(0, std::atoi(need().c_str()));
    } else if (a == "--oracle") {
      o->oracle = need();
    } else if (a == "--perturb-oracle") {
      o->perturb_oracle = std::atof(need().c_str());
    } else {
      return false;
    }
  }
  return o->B > 0 && o->H > 0 && o->N > 0 && o->D > 0;
}

// splitmix64 (Steele, Lea and Flood, 2014) as a seeded uniform source; Box-Muller for N(0, 1).
struct Normal {
  uint64_t state;
  explicit Normal(uint64_t seed) : state(seed * 0x9E3779B97F4A7C15ull + 1) {}
  uint64_t next() {
    uint64_t z = (state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  double uniform() { return (static_cast<double>(next() >> 11) + 0.5) * 0x1.0p-53; }
  void pair(float* a, float* b) {
    const double r = std::sqrt(-2.0 * std::log(uniform()));
    const double t = 6.283185307179586 * uniform();
    *a = static_cast<float>(r * std::cos(t));
    *b = static_cast<float>(r * std::sin(t));
  }
};

// n values rounded to the kernel dtype: 16-bit words for the device, doubles for the oracle.
void make_input(Normal& g, size_t n, int dtype, std::vector<uint16_t>* bits,
                std::vector<double>* wide) {
  bits->resize(n);
  wide->resize(n);
  for (size_t i = 0; i < n; i += 2) {
    float x[2];
    g.pair(&x[0], &x[1]);
    for (size_t j = 0; j < 2 && i + j < n; ++j) {
      uint16_t w;
      double d;
      if (dtype == FA_DTYPE_BF16) {
        const __nv_bfloat16 h = __float2bfloat16_rn(x[j]);
        std::memcpy(&w, &h, 2);
        d = static_cast<double>(__bfloat162float(h));
      } else {
        const __half h = __float2half_rn(x[j]);
        std::memcpy(&w, &h, 2);
        d = static_cast<double>(__half2float(h));
      }
      (*bits)[i + j] = w;
      (*wide)[i + j] = d;
    }
  }
}

double to_double(uint16_t w, int dtype) {
  if (dtype == FA_DTYPE_BF16) {
    __nv_bfloat16 h;
    std::memcpy(&h, &w, 2);
    return static_cast<double>(__bfloat162float(h));
  }
  __half h;
  std::memcpy(&h, &w, 2);
  return static_cast<double>(__half2float(h));
}

std::string default_oracle_path(const char* argv0) {
  // <repo>/fused-attention-cuda_b200/fused_attn/fa_bench -> <repo>/oracle/libfa_oracle.so
  std::string p = argv0;
  const size_t cut = p.rfind('/');
  const std::string dir = cut == std::string::npos ? "." : p.substr(0, cut);
  return dir + "/../../oracle/libfa_oracle.so";
}

double percentile(std::vector<double> v, double q) {
  std::sort(v.begin(), v.end());
  const size_t i = static_cast<size_t>(std::lround(q * static_cast<double>(v.size() - 1)));
  return v[std::min(i, v.size() - 1)];
}

}  // namespace

int main(int argc, char** argv) {
  Options opt;
  if (!parse(argc, argv, &opt)) {
    std::fprintf(stderr,
                 "usage: fa_bench [--cfg B2_H8_N2048_D128] [--dtype fp16|bf16] [--causal 0|1] "
                 "[--seed S] [--iters K] [--warmup W] [--oracle PATH] [--threads T]\n");
    return 1;
  }
  if (opt.oracle.empty()) opt.oracle = default_oracle_path(argv[0]);
  if (opt.threads == 0) opt.threads = std::max(1u, std::thread::hardware_concurrency());
  const int B = opt.B, H = opt.H, N = opt.N, D = opt.D;
  const size_t n_elem = static_cast<size_t>(B) * H * N * D;
  const size_t n_rows = static_cast<size_t>(B) * H * N;
  const double scale = 1.0 / std::sqrt(static_cast<double>(D));

  // ---- inputs (q, k, v in that order from one seeded stream) --------------------------------
  Normal gen(opt.seed);
  std::vector<uint16_t> hq, hk, hv;
  std::vector<double> wq, wk, wv;
  make_input(gen, n_elem, opt.dtype, &hq, &wq);
  make_input(gen, n_elem, opt.dtype, &hk, &wk);
  make_input(gen, n_elem, opt.dtype, &hv, &wv);

  void *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *flush = nullptr;
  float* lse = nullptr;
  const size_t bytes = n_elem * 2;
  const size_t flush_bytes = 256ull << 20;
  if (!check(cudaMalloc(&q, bytes), "cudaMalloc q") || !check(cudaMalloc(&k, bytes), "cudaMalloc k") ||
      !check(cudaMalloc(&v, bytes), "cudaMalloc v") || !check(cudaMalloc(&o, bytes), "cudaMalloc o") ||
      !check(cudaMalloc(&lse, n_rows * 4), "cudaMalloc lse") ||
      !check(cudaMalloc(&flush, flush_bytes), "cudaMalloc flush")) {
    return 1;
  }
  if (!check(cudaMemcpy(q, hq.data(), bytes, cudaMemcpyHostToDevice), "copy q") ||
      !check(cudaMemcpy(k, hk.data(), bytes, cudaMemcpyHostToDevice), "copy k") ||
      !check(cudaMemcpy(v, hv.data(), bytes, cudaMemcpyHostToDevice), "copy v")) {
    return 1;
  }
  cudaStream_t stream;
  if (!check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream")) return 1;
  const fa_params_t p{B, H, H, N, D, static_cast<float>(scale), opt.causal};

  // ---- pre-flight ------------------------------------------------------------------------------
  int rc = fa_forward(FA_IMPL_TUNED, opt.dtype, q, k, v, o, lse, nullptr, &p, stream);
  if (rc != 0) {
    std::fprintf(stderr, "fa_bench: fa_forward returned %d (%s)\n", rc,
                 cudaGetErrorString(static_cast<cudaError_t>(rc)));
    return 1;
  }
  unsigned int detail = 0;
  rc = fa_last_device_error(&detail);  // synchronises the device
  if (rc != 0) {
    std::fprintf(stderr, "fa_bench: device status %d (bits 0x%x)\n", rc, detail);
    return 1;
  }

  // ---- self-check against the fp64 oracle: heads (0, 0) and (B-1, H-1) in full -----------------
  void* so = dlopen(opt.oracle.c_str(), RTLD_NOW | RTLD_LOCAL);
  if (so == nullptr) {
    std::fprintf(stderr, "fa_bench: cannot load the oracle %s: %s (no row without a check)\n",
                 opt.oracle.c_str(), dlerror());
    return 2;
  }
  auto oracle = reinterpret_cast<OracleAttentionFn>(dlsym(so, "fa_oracle_attention"));
  if (oracle == nullptr) {
    std::fprintf(stderr, "fa_bench: fa_oracle_attention missing in %s\n", opt.oracle.c_str());
    return 2;
  }
  std::vector<uint16_t> ho(n_elem);
  std::vector<float> hl(n_rows);
  if (!check(cudaMemcpy(ho.data(), o, bytes, cudaMemcpyDeviceToHost), "copy o") ||
      !check(cudaMemcpy(hl.data(), lse, n_rows * 4, cudaMemcpyDeviceToHost), "copy lse")) {
    return 1;
  }
  const double tol_o = opt.dtype == FA_DTYPE_BF16 ? 8e-3 : 2e-3, tol_lse = 1e-3;
  double err_o = 0.0, err_lse = 0.0;
  const size_t head = static_cast<size_t>(N) * D;
  const OracleShape one{1, 1, 1, N, D, scale, opt.causal};
  const int heads[2][2] = {{0, 0}, {B - 1, H - 1}};
  for (int c = 0; c < (B * H > 1 ? 2 : 1); ++c) {
    const size_t bh = static_cast<size_t>(heads[c][0]) * H + heads[c][1];
    std::vector<double> ro(head), rl(N);
    // fa_oracle_attention returns the number of threads it ran on (at least 1).
    if (oracle(wq.data() + bh * head, wk.data() + bh * head, wv.data() + bh * head, &one, ro.data(),
               rl.data(), opt.threads) < 1) {
      std::fprintf(stderr, "fa_bench: the oracle failed\n");
      return 2;
    }
    for (size_t i = 0; i < head; ++i) {
      const double e = std::fabs(to_double(ho[bh * head + i], opt.dtype) - (ro[i] + opt.perturb_oracle));
      if (!(e <= err_o)) err_o = std::isnan(e) ? INFINITY : e;
    }
    for (int r = 0; r < N; ++r) {
      const double e = std::fabs(static_cast<double>(hl[bh * N + r]) - rl[r]);
      if (!(e <= err_lse)) err_lse = std::isnan(e) ? INFINITY : e;
    }
  }
  const bool passed = err_o <= tol_o && err_lse <= tol_lse;
  if (!passed) {
    std::fprintf(stderr,
                 "fa_bench: self-check FAILED (max|dO| %.3e > %.1e or max|dLSE| %.3e > %.1e): "
                 "row refused\n",
                 err_o, tol_o, err_lse, tol_lse);
    return 2;
  }

  // ---- timed loop: memset flush, event, launch, event; one synchronisation at the end ---------
  for (int i = 0; i < opt.warmup; ++i) {
    cudaMemsetAsync(flush, 0, flush_bytes, stream);
    fa_forward(FA_IMPL_TUNED, opt.dtype, q, k, v, o, lse, nullptr, &p, stream);
  }
  std::vector<cudaEvent_t> ev(2 * static_cast<size_t>(opt.iters));
  for (auto& e : ev) {
    if (!check(cudaEventCreate(&e), "event")) return 1;
  }
  for (int i = 0; i < opt.iters; ++i) {
    cudaMemsetAsync(flush, 0, flush_bytes, stream);
    cudaEventRecord(ev[2 * i], stream);
    rc = fa_forward(FA_IMPL_TUNED, opt.dtype, q, k, v, o, lse, nullptr, &p, stream);
    cudaEventRecord(ev[2 * i + 1], stream);
    if (rc != 0) break;
  }
  if (!check(cudaStreamSynchronize(stream), "sync")) return 1;
  if (rc != 0) {
    std::fprintf(stderr, "fa_bench: fa_forward returned %d in the timed loop\n", rc);
    return 1;
  }
  rc = fa_last_device_error(&detail);
  if (rc != 0) {
    std::fprintf(stderr, "fa_bench: device status %d (bits 0x%x) after timing\n", rc, detail);
    return 1;
  }
  std::vector<double> ms(opt.iters);
  for (int i = 0; i < opt.iters; ++i) {
    float t = 0.f;
    cudaEventElapsedTime(&t, ev[2 * i], ev[2 * i + 1]);
    ms[i] = t;
  }
  const double flops = 4.0 * B * H * static_cast<double>(N) * N * D / (opt.causal ? 2.0 : 1.0);
  const double med = percentile(ms, 0.5);
  std::printf(
      "{\"harness\": \"fa_bench\", \"cfg\": \"B%d_H%d_N%d_D%d\", \"dtype\": \"%s\", \"causal\": %d, "
      "\"iters\": %d, \"warmup\": %d, \"median_ms\": %.6f, \"p10_ms\": %.6f, \"p90_ms\": %.6f, "
      "\"tflops\": %.3f, \"l2_flush_bytes\": %zu, \"self_check\": {\"passed\": true, "
      "\"heads\": [[0, 0], [%d, %d]], \"max_abs_o\": %.3e, \"max_abs_lse\": %.3e, "
      "\"oracle\": \"%s\", \"threads\": %d}}\n",
      B, H, N, D, fa_dtype_name(opt.dtype), opt.causal, opt.iters, opt.warmup, med,
      percentile(ms, 0.1), percentile(ms, 0.9), flops / (med * 1e-3) / 1e12, flush_bytes, B - 1,
      H - 1, err_o, err_lse, opt.oracle.c_str(), opt.threads);
  for (auto& e : ev) cudaEventDestroy(e);
  cudaStreamDestroy(stream);
  cudaFree(q);
  cudaFree(k);
  cudaFree(v);
  cudaFree(o);
  cudaFree(lse);
  cudaFree(flush);
  dlclose(so);
  return 0;
}
