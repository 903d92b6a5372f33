// fa_kernel_common.cuh -- device-side pieces shared by the sm_100a SDPA forward kernels:
// the launch-wide status words, work-item order, bounded mbarrier waits and the softmax row
// primitives.  Included by exactly one translation unit (fa_fwd_sm100.cu), so the __device__
// status words below have one definition that the host reads back.
#pragma once

#include <cmath>
#include <type_traits>

#include "fa_launch.h"
#include "sm100_ptx.cuh"

namespace fa_sm100 {

__device__ unsigned int g_status;       // sticky cause bits of timed-out waits
__device__ unsigned int g_abort_epoch;  // epoch of the last launch in which a wait ran out

#ifdef FA_TRACE
// Debug builds only: SM-clock timestamps of the first item of the first kTraceCtas CTAs, per
// event kind e (0 S issued, 1 PV issued, 2 S seen by softmax, 3 P stored), group g, tile t.
constexpr int kTraceCtas = 8, kTraceTiles = 64;
__device__ long long g_trace[kTraceCtas][6][2][kTraceTiles];
__device__ long long g_trace_t0[kTraceCtas];
#define FA_TRACE_EV(first, e, g, t)                                                      \
  do {                                                                                   \
    if ((first) && blockIdx.x < kTraceCtas && (t) < kTraceTiles)                         \
      g_trace[blockIdx.x][e][g][t] = clock64() - g_trace_t0[blockIdx.x];                 \
  } while (0)
#else
#define FA_TRACE_EV(first, e, g, t) \
  do {                              \
  } while (0)
#endif

// FA_DEBUG_CHECKS builds (-DFA_DEBUG_CHECKS; build.py makes libfa_sm100_checks.so): index and
// address checks in front of the kernels' computed accesses -- tensor-memory columns against the
// allocation, shared-memory offsets against the layout, global LSE / O / workspace indices
// against the tensor sizes, work items against the item count.  A failed check sets kStBounds in
// g_status (fa_last_device_error then returns cudaErrorAssert) and the guarded access is skipped:
// nothing traps, the kernel runs on, and its bounded waits end any hand-off the skip disturbs.
// Release builds compile every check to `true`.
#ifdef FA_DEBUG_CHECKS
#define FA_DCHECK(cond) ((cond) ? true : (atomicOr(&g_status, kStBounds), false))
#else
#define FA_DCHECK(cond) true
#endif

namespace {

constexpr int kBlockM = 128;
constexpr int kThreads = 384;
constexpr int kSoftmaxWarp0 = 4;  // warps 4..11: two softmax warpgroups
constexpr int kMergeBarrier = 1;  // named barrier id shared by the 256 softmax threads
constexpr float kRescaleThreshold = 8.0f;

struct KArgs {
  void* o;
  long long o_sb, o_sh, o_sn;  // element strides of o's (b, h, n) dimensions (d is contiguous)
  float* lse;                  // [B, H, N] contiguous
  int q_pos, k_pos, v_pos;     // tensor-map dimension (2 bits each) holding n, h, b
  int o_pos;                   // the same for the output map (kernels that store O by TMA)
  int H, Hkv, N;
  int n_q_tiles;
  int n_bh;        // B * H
  int n_items;     // n_bh * n_q_tiles work items (one 128-row query tile of one head each)
  int head_group;  // heads per scheduling group (K/V of one group stays in L2)
  float scale;
  float scale_log2;
  unsigned long long timeout_ns;
  unsigned int epoch;
  int skip_kv_tile;
};

// Work items are visited in a fixed order and dealt to the persistent CTAs boustrophedon-wise:
// round r gives item r*G + c to CTA c on even rounds and r*G + (G-1-c) on odd ones, which pairs
// heavy with light items across rounds.  The order walks the heads in groups whose K/V fits in
// L2 (all heads at once when it all fits); inside a group, heaviest causal query tiles first
// (longest processing time first), the group's heads interleaved under each query tile.
struct Item {
  int bh, q_tile;
};

// (batch, query head, kv head) of flattened head index bh = b * H + h.
struct Heads {
  int b, h, hk;
};
__device__ __forceinline__ Heads split_heads(int bh, const KArgs& a) {
  const int b = bh / a.H;
  const int h = bh - b * a.H;
  return Heads{b, h, h / (a.H / a.Hkv)};
}

// TMA load of one box of a [b][h][n][d] view whose map orders n, h, b by stride (`pos`).
__device__ __forceinline__ void tma_load_view(uint32_t dst, const void* tmap, int x, int n, int h,
                                              int b, int pos, uint32_t bar) {
  const int pn = pos & 3, ph = (pos >> 2) & 3;
  const int c0 = pn == 0 ? n : (ph == 0 ? h : b);
  const int c1 = pn == 1 ? n : (ph == 1 ? h : b);
  const int c2 = pn == 2 ? n : (ph == 2 ? h : b);
  tma_load_4d(dst, tmap, x, c0, c1, c2, bar);
}

// TMA store of one box from shared memory into the [b][h][n][d] view of O (same coordinate
// order as tma_load_view).
__device__ __forceinline__ void tma_store_view(const void* tmap, uint32_t src, int x, int n, int h,
                                               int b, int pos) {
  const int pn = pos & 3, ph = (pos >> 2) & 3;
  const int c0 = pn == 0 ? n : (ph == 0 ? h : b);
  const int c1 = pn == 1 ? n : (ph == 1 ? h : b);
  const int c2 = pn == 2 ? n : (ph == 2 ? h : b);
  tma_store_4d(tmap, x, c0, c1, c2, src);
}

// First element of output row `row` of head bh.
template <typename T>
__device__ __forceinline__ T* out_row(const KArgs& a, int bh, int row) {
  const Heads hd = split_heads(bh, a);
  return reinterpret_cast<T*>(a.o) + hd.b * a.o_sb + hd.h * a.o_sh +
         static_cast<long long>(row) * a.o_sn;
}

__device__ __forceinline__ int item_index(int round, int G, int c) {
  return round * G + ((round & 1) ? (G - 1 - c) : c);
}

template <bool CAUSAL>
__device__ __forceinline__ Item decode_item(int i, const KArgs& a) {
  const int per_group = a.head_group * a.n_q_tiles;
  const int k = i / per_group;                           // head group
  const int j = i - k * per_group;                       // index inside the group
  const int hg = min(a.head_group, a.n_bh - k * a.head_group);  // heads in this group
  const int qr = j / hg;
  const int bh = k * a.head_group + (j - qr * hg);
  return Item{bh, CAUSAL ? a.n_q_tiles - 1 - qr : qr};
}

struct WaitCtx {
  volatile int* abort_flag;
  unsigned long long timeout_ns;
  unsigned int epoch;
};

// Bounded wait: true when the phase completed; false when this CTA aborts (own time limit,
// another role of this CTA gave up, or another CTA of this launch gave up).
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, const WaitCtx& w,
                                             unsigned int cause) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*w.abort_flag) return false;
    if (globaltimer_ns() - t0 > w.timeout_ns) {
      *w.abort_flag = 1;
      atomicOr(&g_status, cause);
      atomicExch(&g_abort_epoch, w.epoch);
      return false;
    }
    if ((++spins & 63u) == 0u &&
        *reinterpret_cast<volatile unsigned int*>(&g_abort_epoch) == w.epoch) {
      *w.abort_flag = 1;
      return false;
    }
  }
}

// Exit-path wait for this CTA's own in-flight work (copies / MMAs); ignores the abort flag but is
// still bounded.
__device__ __forceinline__ void wait_drain(uint32_t bar, uint32_t parity,
                                           unsigned long long timeout_ns) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      atomicOr(&g_status, kStDrain);
      return;
    }
  }
}

// Every kEmuEvery-th pair of exponentials goes to the FMA pipes (ex2_poly3) instead of the MUFU
// unit; 0 keeps them all on MUFU.  Set at build time with -DFA_EX2_EMU_EVERY=n.  One pair in eight
// measured best for the 128-key kernel (the D=64 full-attention default): B2H8 N8192 D64 664 ->
// 692 TFLOP/s, B8H32 N2048 608 -> 620, C2 418 -> 419; one in six or four is slower.
#ifndef FA_EX2_EMU_EVERY
#define FA_EX2_EMU_EVERY 8
#endif
constexpr int kEmuEvery = FA_EX2_EMU_EVERY;

// Loads one S row (BN fp32 columns of this thread's TMEM lane) with one instruction.
template <int BN>
__device__ __forceinline__ void load_s_row(uint32_t taddr, float (&s)[BN]) {
  uint32_t u[BN];
  if constexpr (BN == 128) {
    tmem_ld128_wait(taddr, u);
  } else if constexpr (BN == 64) {
    tmem_ld64_wait(taddr, u);
  } else {
    tmem_ld32_wait(taddr, u);
  }
#pragma unroll
  for (int i = 0; i < BN; ++i) s[i] = __uint_as_float(u[i]);
}

// Row maximum with eight independent three-input max chains (BN/16 deep instead of BN).
template <int BN>
__device__ __forceinline__ float row_max(const float (&s)[BN]) {
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = fmaxf(s[2 * k], s[2 * k + 1]);
#pragma unroll
  for (int i = 16; i < BN; i += 16) {
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = fmax3(a[k], s[i + 2 * k], s[i + 2 * k + 1]);
  }
  return fmax3(fmax3(a[0], a[1], a[2]), fmax3(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
}

// p = 2^(s*c - m*c) for columns [2*C0, 2*C1) of one S row: the exponent argument in packed fp32
// pairs, the exponential on MUFU (every kEmuEvery-th pair on the FMA pipes), P packed two per
// 32-bit word and stored to TMEM at `taddr` + C0 (one column per pair), sixteen columns at a time
// as they are computed (eight with P_lo) so that only sixteen packed words are live.  Returns the
// sum of the fp32 weights, accumulated in four packed partial sums.  kLo (bf16 only) also stores
// P_lo = p - bf16(p) at `taddr` + BN/2 + C0.
template <typename T, int BN, int C0, int C1, bool kLo>
__device__ __forceinline__ float exp_pack_store(const float (&s)[BN], float sl2, float mc,
                                                uint32_t taddr) {
  static_assert((C1 - C0) % 16 == 0, "column range must be a multiple of 16 pairs");
  constexpr int kN = C1 - C0;
  constexpr int kChunk = kLo ? 8 : 16;
  const uint64_t c2 = f2_pack(sl2, sl2);
  const uint64_t nb2 = f2_pack(-mc, -mc);
  uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int c0 = 0; c0 < kN; c0 += kChunk) {
    uint32_t pk[kChunk];
    uint32_t lo[kLo ? kChunk : 1];
#pragma unroll
    for (int c = 0; c < kChunk; ++c) {
      const int cc = C0 + c0 + c;
      const uint64_t x = f2_fma(f2_pack(s[2 * cc], s[2 * cc + 1]), c2, nb2);
      float p0, p1;
      if (kEmuEvery > 0 && (cc % (kEmuEvery > 0 ? kEmuEvery : 1)) == (kEmuEvery > 0 ? kEmuEvery : 1) - 1) {
        p0 = ex2_poly3(f2_lo(x));
        p1 = ex2_poly3(f2_hi(x));
      } else {
        p0 = ex2_approx(f2_lo(x));
        p1 = ex2_approx(f2_hi(x));
      }
      pk[c] = pack2<T>(p0, p1);
      acc[c & 3] = f2_add(acc[c & 3], f2_pack(p0, p1));
      if constexpr (kLo) {
        lo[c] = pack2<T>(p0 - __uint_as_float(pk[c] << 16), p1 - __uint_as_float(pk[c] & 0xFFFF0000u));
      }
    }
    if constexpr (kLo) {
      tmem_st8(taddr + C0 + c0, pk);
      tmem_st8(taddr + BN / 2 + C0 + c0, lo);
    } else {
      tmem_st16(taddr + C0 + c0, pk);
    }
  }
  const uint64_t t = f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
  return f2_lo(t) + f2_hi(t);
}

// fp32 flavour for the tf32 path: p = 2^(s*c - m*c) for all BN columns, stored one weight per
// TMEM column (rounded to tf32, the precision the tensor core multiplies) over S_g itself.
// Returns the sum of the unrounded weights.
template <int BN>
__device__ __forceinline__ float exp_store_f32(const float (&s)[BN], float sl2, float mc,
                                               uint32_t taddr) {
  const uint64_t c2 = f2_pack(sl2, sl2);
  const uint64_t nb2 = f2_pack(-mc, -mc);
  uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int c0 = 0; c0 < BN; c0 += 32) {
    uint32_t w32[32];
#pragma unroll
    for (int c = 0; c < 32; c += 2) {
      const uint64_t x = f2_fma(f2_pack(s[c0 + c], s[c0 + c + 1]), c2, nb2);
      const float p0 = ex2_approx(f2_lo(x));
      const float p1 = ex2_approx(f2_hi(x));
      w32[c] = f32_to_tf32(p0);
      w32[c + 1] = f32_to_tf32(p1);
      acc[(c >> 1) & 3] = f2_add(acc[(c >> 1) & 3], f2_pack(p0, p1));
    }
    tmem_st32(taddr + c0, w32);
  }
  const uint64_t t = f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
  return f2_lo(t) + f2_hi(t);
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace
}  // namespace fa_sm100
