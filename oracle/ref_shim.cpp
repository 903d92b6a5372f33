// ref_shim.cpp -- extern "C" entry points over the reference's OWN fp64 oracle.
// TEST INFRASTRUCTURE ONLY (see oracle/fa_oracle.c for who may load it).
//
// This file is compiled together with the reference's unmodified
// src/reference/cpu_reference.cpp, where it lies (oracle/Makefile, target `ref`), into
// oracle/_ref/libfa_ref.so.  Nothing from the reference is copied into this repository: the
// shim only declares flat C signatures that ctypes can bind and forwards them to
//   fa::ref::attention_rows   (src/reference/cpu_reference.h:31-34)
//   fa::ref::attention        (src/reference/cpu_reference.h:36-38)
//   fa::ref::attention_tiled  (src/reference/cpu_reference.h:44-46)
// The threaded driver splits (b, h) heads over std::thread, one attention_rows call per head
// slice, the way the reference's own CPU timing harness parallelises its oracle.
#include <algorithm>
#include <atomic>
#include <thread>
#include <vector>

#include "cpu_reference.h"

namespace {

fa::ref::Shape make_shape(int B, int H, int Hkv, int N, int D, double scale, int causal) {
  fa::ref::Shape s;
  s.B = B, s.H = H, s.Hkv = Hkv, s.N = N, s.D = D, s.scale = scale, s.causal = causal != 0;
  return s;
}

}  // namespace

extern "C" {

// Whole tensor through fa::ref::attention_rows on `threads` threads; returns threads used.
int fa_ref_attention(const double* q, const double* k, const double* v, int B, int H, int Hkv,
                     int N, int D, double scale, int causal, double* o, double* lse,
                     int threads) {
  const fa::ref::Shape s = make_shape(B, H, Hkv, N, D, scale, causal);
  const int row_block = 64;
  const int blocks = (N + row_block - 1) / row_block;
  const long long items = static_cast<long long>(B) * H * blocks;
  std::atomic<long long> next{0};
  auto run = [&] {
    for (;;) {
      const long long it = next.fetch_add(1);
      if (it >= items) return;
      const int blk = static_cast<int>(it % blocks);
      const long long bh = it / blocks;
      const int b = static_cast<int>(bh / H), h = static_cast<int>(bh % H);
      const int row0 = blk * row_block;
      const int rows = std::min(row_block, N - row0);
      double* ob = o + ((static_cast<size_t>(bh) * N) + row0) * D;
      double* lb = lse ? lse + static_cast<size_t>(bh) * N + row0 : nullptr;
      fa::ref::attention_rows(q, k, v, s, b, h, row0, rows, ob, lb);
    }
  };
  threads = std::max(1, std::min<int>(threads, static_cast<int>(std::max<long long>(items, 1))));
  if (threads == 1) {
    run();
    return 1;
  }
  std::vector<std::thread> pool;
  pool.reserve(threads);
  for (int t = 0; t < threads; ++t) pool.emplace_back(run);
  for (auto& t : pool) t.join();
  return threads;
}

// Rows [row0, row0+rows) of head (b, h): o is rows*D, lse rows (or NULL).
void fa_ref_rows(const double* q, const double* k, const double* v, int B, int H, int Hkv, int N,
                 int D, double scale, int causal, int b, int h, int row0, int rows, double* o,
                 double* lse) {
  const fa::ref::Shape s = make_shape(B, H, Hkv, N, D, scale, causal);
  fa::ref::attention_rows(q, k, v, s, b, h, row0, rows, o, lse);
}

// The reference's tiled online-softmax model.
void fa_ref_attention_tiled(const double* q, const double* k, const double* v, int B, int H,
                            int Hkv, int N, int D, double scale, int causal, int block_m,
                            int block_n, double* o, double* lse) {
  const fa::ref::Shape s = make_shape(B, H, Hkv, N, D, scale, causal);
  fa::ref::attention_tiled(q, k, v, s, block_m, block_n, o, lse);
}

}  // extern "C"
