// fa_fwd_sm100.cu -- fused scaled-dot-product-attention forward for B200 (sm_100a).
//
// Replaces the reference's hot kernel fa_s5_tuned / attention_block
// (src/stage5_tuned.cu:450-749) and its host launcher (src/stage5_tuned.cu:802-1037) with a
// Blackwell-native design.  The numerics are the reference's recurrence
// (include/fa/softmax_math.cuh:1-73): running max m in RAW score units, c = scale*log2(e),
// p = 2^(s*c - m*c), alpha = 2^((m_old - m_new)*c), l = alpha*l + sum(p), acc = alpha*acc + P V,
// o = acc * (1/l), lse = m*scale + ln(l), with the empty-row guards (o = 0, lse = +inf).
// Top-left causal: key tiles past the query tile's last row are never loaded
// (stage5_tuned.cu:532-533); the diagonal tile is masked element-wise (:596-602).
//
// One CTA computes one 128-row query tile of one (batch, head).  Warp roles (384 threads):
//   warp 0      TMA producer: Q once, then K_j / V_j through a STAGES-deep shared-memory ring
//               (full/empty mbarrier pairs; K and V have separate slots so K_{j+STAGES} can land
//               while V_j is still being read).
//   warp 1      owns tensor memory (alloc/dealloc); lane 0 issues every tcgen05.mma.
//   warps 2-3   idle (they only join the final barrier).
//   warps 4-7   softmax warpgroup 0: key tiles j = 0, 2, 4, ...
//   warps 8-11  softmax warpgroup 1: key tiles j = 1, 3, 5, ...
// Each softmax warpgroup runs its own online softmax (own running max m_w and sums l_w) over its
// half of the key tiles into its own accumulator O_w; one thread per query row (TMEM lane = row).
// The two partial results are merged at the end exactly like two split-KV partials:
//   m = max(m0, m1), a_w = 2^((m_w - m) c), l = a0 l0 + a1 l1, o = (a0 O0 + a1 O1) / l.
// Splitting the key tiles (instead of giving each warpgroup its own 128 query rows) keeps the
// work item at 128 rows, which keeps causal workloads balanced across the 148 SMs.
//
// Tensor memory (128 lanes = 128 query rows; columns): S_0 [0, BN), S_1 [BN, 2BN),
// O_0 [2BN, 2BN+D), O_1 [2BN+D, 2BN+2D).  P_w (16-bit, BN/2 columns) is written over the first
// half of S_w once the S row is in registers, and is the A operand of the TS-MMA O_w += P_w V_j.
// MMA issue order: S_0(0), S_1(0), then per round t: PV_0(t), S_0(t+1), PV_1(t), S_1(t+1), with
//   S_w(t)   = Q K_{2t+w}^T          (SS: Q and K in smem, K-major, 128-byte swizzle)
//   PV_w(t)  : O_w += P_w V_{2t+w}   (TS: P from TMEM, V from smem as an MN-major operand)
// so the tensor core works for one warpgroup while the other runs its softmax.  S_w(t+1)
// overwrites the columns PV_w(t) reads right after it; tcgen05.mma instructions issued by one
// thread execute in issue order, so the reads come first (FlashAttention-4's forward relies on
// the same order).  The commit of S_w(t+1) covers every earlier MMA, so a softmax warpgroup that
// sees S_w(t+1) complete also knows PV_w(t) is complete before it rescales O_w.
//
// bf16 keeps 8 significant bits.  Rows of the first causal query tile average only a handful of
// keys, where rounding P to bf16 would add up to ~2^-9 |v| to the output's own rounding; there P
// is carried as P_hi + P_lo (both bf16, the second half of S_w holds P_lo) and multiplied twice.
// Every other row averages >= 128 keys and its rounding errors average out.

// O rescaling is lazy: the max used for the exponent (m_ref) only moves when the tile max
// exceeds it by more than 2^8 in exponent units, so P stays <= 256 (exact in fp16/bf16 range)
// and the O read-modify-write through TMEM is rare.  The final o = acc/l and lse use the same
// m_ref, so the result is the same function (FlashAttention-4's conditional rescaling).
//
// Every mbarrier wait is bounded (globaltimer); a wait that runs out sets a CTA-local abort flag,
// records a cause bit in g_status and the launch epoch in g_abort_epoch (so other CTAs of the
// same launch stop early), then the CTA drains its own TMA copies and MMAs, frees TMEM and exits.
// Named barriers are always reached by all of their threads, on the abort path too.
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <type_traits>

#include <atomic>

#include "fa_launch.h"
#include "fa_sm100.h"
#include "sm100_ptx.cuh"

namespace fa_sm100 {

__device__ unsigned int g_status;       // sticky cause bits of timed-out waits
__device__ unsigned int g_abort_epoch;  // epoch of the last launch in which a wait ran out

namespace {

constexpr int kBlockM = 128;
constexpr int kThreads = 384;
constexpr int kSoftmaxWarp0 = 4;  // warps 4..11: two softmax warpgroups
constexpr int kMergeBarrier = 1;  // named barrier id shared by the 256 softmax threads
constexpr float kRescaleThreshold = 8.0f;

template <int D, int BN, int STAGES>
struct Layout {
  static constexpr int kEB = 2;                  // bytes per element (fp16/bf16)
  static constexpr int kSwElems = 128 / kEB;     // elements per 128-byte swizzle row
  static constexpr int kDChunks = D / kSwElems;  // 128-byte column chunks along D
  static constexpr int kQChunkBytes = kBlockM * 128;
  static constexpr int kKVChunkBytes = BN * 128;
  static constexpr int kQBytes = kBlockM * D * kEB;
  static constexpr int kKVBytes = BN * D * kEB;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + STAGES * kKVBytes;
  static constexpr int kBarOff = kVOff + STAGES * kKVBytes;
  static constexpr int kNumBars = 8 + 4 * STAGES;
  static constexpr int kMiscOff = kBarOff + 8 * kNumBars;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kSmemAlloc = kBytes + 1024;  // slack to align the base to 1024 bytes

  // Tensor memory columns.
  static constexpr int kColS = 0;       // + w * BN
  static constexpr int kColO = 2 * BN;  // + w * D
  static constexpr int kColsUsed = 2 * BN + 2 * D;
  static constexpr int kTmemCols = kColsUsed <= 32    ? 32
                                   : kColsUsed <= 64  ? 64
                                   : kColsUsed <= 128 ? 128
                                   : kColsUsed <= 256 ? 256
                                                      : 512;

  // Barrier indices.
  static constexpr int kBarQ = 0;
  static constexpr int kBarKFull = 1;                // + stage
  static constexpr int kBarVFull = 1 + STAGES;       // + stage
  static constexpr int kBarKEmpty = 1 + 2 * STAGES;  // + stage
  static constexpr int kBarVEmpty = 1 + 3 * STAGES;  // + stage
  static constexpr int kBarSFull = 1 + 4 * STAGES;   // + warpgroup
  static constexpr int kBarPFull = 3 + 4 * STAGES;   // + warpgroup
  static constexpr int kBarPVDone = 5 + 4 * STAGES;  // + warpgroup
  static constexpr int kBarDrain = 7 + 4 * STAGES;

  // The merge exchange (m, l per row and warpgroup) reuses the Q tile once every MMA is done.
  static constexpr int kMergeFloats = 2 * 2 * kBlockM;
  static_assert(kMergeFloats * 4 <= kQBytes, "merge exchange must fit in the Q tile");
  static_assert(D % kSwElems == 0, "D must be a multiple of the swizzle width");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 128, "BN must be 32, 64 or 128");
  static_assert(kColsUsed <= 512, "tensor memory overflow");
  static_assert(kSmemAlloc <= 232448, "shared memory overflow");
};

struct KArgs {
  void* o;
  float* lse;
  int H, Hkv, N;
  int n_q_tiles;
  int head_major;  // 1: consecutive CTAs walk the query tiles of one head (L2 reuse of K/V)
  float scale;
  float scale_log2;
  unsigned long long timeout_ns;
  unsigned int epoch;
  int skip_kv_tile;
};

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
// unit; 0 keeps them all on MUFU.  Set at build time with -DFA_EX2_EMU_EVERY=n.
#ifndef FA_EX2_EMU_EVERY
#define FA_EX2_EMU_EVERY 0
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

// Row maximum with four independent three-input max chains (BN/8 deep instead of BN).
template <int BN>
__device__ __forceinline__ float row_max(const float (&s)[BN]) {
  float a0 = fmaxf(s[0], s[1]), a1 = fmaxf(s[2], s[3]);
  float a2 = fmaxf(s[4], s[5]), a3 = fmaxf(s[6], s[7]);
#pragma unroll
  for (int i = 8; i < BN; i += 8) {
    a0 = fmax3(a0, s[i + 0], s[i + 1]);
    a1 = fmax3(a1, s[i + 2], s[i + 3]);
    a2 = fmax3(a2, s[i + 4], s[i + 5]);
    a3 = fmax3(a3, s[i + 6], s[i + 7]);
  }
  return fmax3(fmaxf(a0, a1), a2, a3);
}

// p = 2^(s*c - m*c) for one S row: the exponent argument in packed fp32 pairs, the exponential
// on MUFU (and every kEmuEvery-th pair on the FMA pipes), P packed two per 32-bit word and stored
// to TMEM at `taddr` (BN/2 columns).  Returns the row sum of the fp32 weights, accumulated in
// four packed partial sums.  kLo (bf16 only) also stores P_lo = p - bf16(p) in the next BN/2
// columns.
template <typename T, int BN, bool kLo>
__device__ __forceinline__ float exp_pack_store(const float (&s)[BN], float sl2, float mc,
                                                uint32_t taddr) {
  const uint64_t c2 = f2_pack(sl2, sl2);
  const uint64_t nb2 = f2_pack(-mc, -mc);
  uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
  uint32_t pk[BN / 2];
  uint32_t lo[kLo ? BN / 2 : 1];
#pragma unroll
  for (int c = 0; c < BN / 2; ++c) {
    const uint64_t x = f2_fma(f2_pack(s[2 * c], s[2 * c + 1]), c2, nb2);
    float p0, p1;
    if (kEmuEvery > 0 && (c % (kEmuEvery > 0 ? kEmuEvery : 1)) == (kEmuEvery > 0 ? kEmuEvery : 1) - 1) {
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
#pragma unroll
  for (int c = 0; c < BN / 2; c += 16) tmem_st16(taddr + c, &pk[c]);
  if constexpr (kLo) {
#pragma unroll
    for (int c = 0; c < BN / 2; c += 16) tmem_st16(taddr + BN / 2 + c, &lo[c]);
  }
  const uint64_t t = f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
  return f2_lo(t) + f2_hi(t);
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <typename T, int D, int BN, int STAGES, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const KArgs args) {
  using L = Layout<D, BN, STAGES>;
  constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  auto bar = [sbase](int i) -> uint32_t { return sbase + L::kBarOff + 8u * i; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Work item: (batch*head, query tile).  Heaviest causal tiles first (longest processing time
  // first keeps the tail short); head-major order when K/V of all heads would not stay in L2.
  int bh, q_tile_rev;
  if (args.head_major) {
    bh = static_cast<int>(blockIdx.x) / args.n_q_tiles;
    q_tile_rev = static_cast<int>(blockIdx.x) % args.n_q_tiles;
  } else {
    const int n_bh = static_cast<int>(gridDim.x) / args.n_q_tiles;
    bh = static_cast<int>(blockIdx.x) % n_bh;
    q_tile_rev = static_cast<int>(blockIdx.x) / n_bh;
  }
  const int q_tile = CAUSAL ? (args.n_q_tiles - 1 - q_tile_rev) : q_tile_rev;
  const int q0 = q_tile * kBlockM;
  const int b_idx = bh / args.H;
  const int h_idx = bh - b_idx * args.H;
  const int bh_kv = b_idx * args.Hkv + h_idx / (args.H / args.Hkv);
  const int kv_end = CAUSAL ? min(args.N, q0 + kBlockM) : args.N;
  const int n_tiles = (kv_end + BN - 1) / BN;  // >= 1
  const int n_t0 = (n_tiles + 1) / 2;          // tiles of warpgroup 0 (even j)
  const int n_t1 = n_tiles / 2;                // tiles of warpgroup 1 (odd j)
  // bf16 keeps 8 significant bits.  In the first causal query tile the rows average only a
  // handful of keys, so rounding P to bf16 would add up to ~2^-9 |v| on top of the output
  // rounding; there P is carried as P_hi + P_lo (two bf16 MMAs).  Everywhere else a row averages
  // >= 128 keys and the rounding errors average out.
  const bool comp = std::is_same<T, __nv_bfloat16>::value && CAUSAL && q_tile == 0;

  if (threadIdx.x == 0) {
    mbar_init(bar(L::kBarQ), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar(L::kBarKFull + s), 1);
      mbar_init(bar(L::kBarVFull + s), 1);
      mbar_init(bar(L::kBarKEmpty + s), 1);
      mbar_init(bar(L::kBarVEmpty + s), 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(bar(L::kBarSFull + g), 1);
      mbar_init(bar(L::kBarPFull + g), kBlockM);
      mbar_init(bar(L::kBarPVDone + g), 1);
    }
    mbar_init(bar(L::kBarDrain), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx w{abort_flag, args.timeout_ns, args.epoch};

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(bar(L::kBarQ), L::kQBytes);
#pragma unroll
      for (int c = 0; c < L::kDChunks; ++c) {
        tma_load_3d(sbase + L::kQOff + c * L::kQChunkBytes, &tm_q, c * L::kSwElems, q0, bh,
                    bar(L::kBarQ));
      }
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = static_cast<uint32_t>(j / STAGES) & 1u;
        if (j >= STAGES && !wait_bounded(bar(L::kBarKEmpty + s), ph ^ 1u, w, kStKVEmpty)) break;
        if (j != args.skip_kv_tile) {
          mbar_arrive_expect_tx(bar(L::kBarKFull + s), L::kKVBytes);
#pragma unroll
          for (int c = 0; c < L::kDChunks; ++c) {
            tma_load_3d(sbase + L::kKOff + s * L::kKVBytes + c * L::kKVChunkBytes, &tm_k,
                        c * L::kSwElems, j * BN, bh_kv, bar(L::kBarKFull + s));
          }
        }
        k_issued = j + 1;
        if (j >= STAGES && !wait_bounded(bar(L::kBarVEmpty + s), ph ^ 1u, w, kStKVEmpty)) break;
        mbar_arrive_expect_tx(bar(L::kBarVFull + s), L::kKVBytes);
#pragma unroll
        for (int c = 0; c < L::kDChunks; ++c) {
          tma_load_3d(sbase + L::kVOff + s * L::kKVBytes + c * L::kKVChunkBytes, &tm_v,
                      c * L::kSwElems, j * BN, bh_kv, bar(L::kBarVFull + s));
        }
        v_issued = j + 1;
      }
      // Exit path: every copy this thread started must have landed before the CTA may exit.
      wait_drain(bar(L::kBarQ), 0u, args.timeout_ns);
      for (int j = (k_issued > STAGES ? k_issued - STAGES : 0); j < k_issued; ++j) {
        if (j != args.skip_kv_tile) {
          wait_drain(bar(L::kBarKFull + j % STAGES), static_cast<uint32_t>(j / STAGES) & 1u,
                     args.timeout_ns);
        }
      }
      for (int j = (v_issued > STAGES ? v_issued - STAGES : 0); j < v_issued; ++j) {
        wait_drain(bar(L::kBarVFull + j % STAGES), static_cast<uint32_t>(j / STAGES) & 1u,
                   args.timeout_ns);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescS = idesc_mma(kFmt, kBlockM, BN, false);
      constexpr uint32_t kIdescPV = idesc_mma(kFmt, kBlockM, D, true);
      // S_g(t) = Q K_j^T, j = 2t + g, into S_g.
      auto issue_s = [&](int g, int t) -> bool {
        const int j = 2 * t + g;
        const int s = j % STAGES;
        if (!wait_bounded(bar(L::kBarKFull + s), static_cast<uint32_t>(j / STAGES) & 1u, w,
                          kStKFull)) {
          return false;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + L::kColS + g * BN;
        const uint32_t kb = sbase + L::kKOff + s * L::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t q_off = (kk / 4) * L::kQChunkBytes + (kk % 4) * 32;
          const uint32_t k_off = (kk / 4) * L::kKVChunkBytes + (kk % 4) * 32;
          umma_ss(d_tmem, sdesc_sw128(sbase + L::kQOff + q_off, 16, 1024),
                  sdesc_sw128(kb + k_off, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar(L::kBarSFull + g));
        umma_commit(bar(L::kBarKEmpty + s));
        return true;
      };
      // O_g += P_g V_j, j = 2t + g.  With `comp` (bf16 causal query tile 0) P_g is two bf16
      // halves P_hi + P_lo in the two halves of S_g, and both are multiplied.
      auto issue_pv = [&](int g, int t, bool last) -> bool {
        const int j = 2 * t + g;
        const int s = j % STAGES;
        if (!wait_bounded(bar(L::kBarPFull + g), static_cast<uint32_t>(t) & 1u, w, kStPFull)) {
          return false;
        }
        if (!wait_bounded(bar(L::kBarVFull + s), static_cast<uint32_t>(j / STAGES) & 1u, w,
                          kStVFull)) {
          return false;
        }
        tc_fence_after();
        const uint32_t vb = sbase + L::kVOff + s * L::kKVBytes;
        const uint32_t pa = tmem + L::kColS + g * BN;
        const uint32_t o_tmem = tmem + L::kColO + g * D;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          umma_ts(o_tmem, pa + kk * 8, sdesc_sw128(vb + kk * 16 * 128, L::kKVChunkBytes, 1024),
                  kIdescPV, (t > 0 || kk > 0) ? 1u : 0u);
        }
        if (comp) {
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            umma_ts(o_tmem, pa + BN / 2 + kk * 8,
                    sdesc_sw128(vb + kk * 16 * 128, L::kKVChunkBytes, 1024), kIdescPV, 1u);
          }
        }
        if (last) umma_commit(bar(L::kBarPVDone + g));
        umma_commit(bar(L::kBarVEmpty + s));
        return true;
      };
      // Issue order PV_0(t), S_0(t+1), PV_1(t), S_1(t+1): while warpgroup 1 runs its softmax the
      // tensor core works for warpgroup 0 and vice versa.  S_g(t+1) overwrites the TMEM columns
      // PV_g(t) reads; tcgen05.mma instructions issued by one thread execute in issue order, so the
      // reads of PV_g(t) precede the writes of S_g(t+1) (FlashAttention-4's forward schedules the
      // same pair the same way).  The commit of S_g(t+1) covers PV_g(t) as well, so a softmax
      // warpgroup that sees S_g(t+1) complete may also rescale O_g.
      bool ok = wait_bounded(bar(L::kBarQ), 0u, w, kStQFull);
      if (ok) ok = issue_s(0, 0);
      if (ok && n_t1 > 0) ok = issue_s(1, 0);
      for (int t = 0; ok && t < n_t0; ++t) {
        if (!(ok = issue_pv(0, t, t + 1 == n_t0))) break;
        if (t + 1 < n_t0 && !(ok = issue_s(0, t + 1))) break;
        if (t < n_t1) {
          if (!(ok = issue_pv(1, t, t + 1 == n_t1))) break;
          if (t + 1 < n_t1 && !(ok = issue_s(1, t + 1))) break;
        }
      }
      // Exit path: all MMAs this thread issued must be complete before TMEM is freed.
      umma_commit(bar(L::kBarDrain));
      wait_drain(bar(L::kBarDrain), 0u, args.timeout_ns);
    }
    __syncwarp();
  } else if (warp >= kSoftmaxWarp0) {
    // ------------------------------------------------------------------ softmax warpgroups
    const int g = (warp - kSoftmaxWarp0) >> 2;  // 0: even key tiles, 1: odd key tiles
    const int n_t = g == 0 ? n_t0 : n_t1;
    const int r = (warp & 3) * 32 + lane;  // row within the tile == TMEM lane
    const int row = q0 + r;
    const uint32_t tl = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_col = L::kColS + g * BN;
    const uint32_t o_col = L::kColO + g * D;
    const float sl2 = args.scale_log2;
    float m_ref = -INFINITY;  // max used in the exponents (raw score units)
    float l_sum = 0.f;        // running sum of the fp32 weights
    bool ok = true;
    for (int t = 0; t < n_t; ++t) {
      const int j = 2 * t + g;
      ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarSFull + g),
                                                static_cast<uint32_t>(t) & 1u, w, kStSFull));
      if (!ok) break;
      tc_fence_after();
      float s[BN];
      load_s_row<BN>(tl + s_col, s);
      const int kv0 = j * BN;
      if ((CAUSAL && kv0 + BN - 1 > q0) || kv0 + BN > args.N) {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const int kv = kv0 + c;
          if (kv >= args.N || (CAUSAL && kv > row)) s[c] = -INFINITY;
        }
      }
      const float m_new = fmaxf(m_ref, row_max<BN>(s));
      const bool resc = (m_ref == -INFINITY) ? (m_new != -INFINITY)
                                             : ((m_new - m_ref) * sl2 > kRescaleThreshold);
      const float m_use = resc ? m_new : m_ref;
      const float alpha =
          resc ? ((m_ref == -INFINITY) ? 0.f : ex2_approx((m_ref - m_use) * sl2)) : 1.f;
      const float mc = (m_use == -INFINITY) ? 0.f : m_use * sl2;
      // P_g over the first half of S_g (all of S_g's row is in registers by now).
      float rs;
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        rs = comp ? exp_pack_store<T, BN, true>(s, sl2, mc, tl + s_col)
                  : exp_pack_store<T, BN, false>(s, sl2, mc, tl + s_col);
      } else {
        rs = exp_pack_store<T, BN, false>(s, sl2, mc, tl + s_col);
      }
      tmem_st_wait();
      l_sum = l_sum * alpha + rs;
      m_ref = m_use;
      // O_g correction.  S_g(t) completing implies PV_g(t-1) completed (the commit of S_g(t)
      // covers every MMA issued before it), and PV_g(t) waits for our arrival below.
      if (t > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          uint32_t u[32];
          tmem_ld32_wait(tl + o_col + c, u);
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
          tmem_st32(tl + o_col + c, u);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive(bar(L::kBarPFull + g));
    }
    // ---- merge the two partials and write O / LSE ------------------------------------------
    if (ok && n_t > 0) {  // committed once, after the warpgroup's last PV
      ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarPVDone + g), 0u, w, kStODone));
    }
    tc_fence_before();
    // Barrier 1: both warpgroups' last PVs are complete, hence every MMA of the CTA is (the last
    // one issued is one of the two), so the Q tile is free for the exchange.
    named_barrier_sync(kMergeBarrier, 256);
    float* xch = reinterpret_cast<float*>(smem + L::kQOff);
    const bool live = (*abort_flag == 0);
    if (live) {
      xch[(g * 2 + 0) * kBlockM + r] = m_ref;
      xch[(g * 2 + 1) * kBlockM + r] = l_sum;
    }
    named_barrier_sync(kMergeBarrier, 256);
    if (live && *abort_flag == 0) {
      tc_fence_after();
      const float m0 = xch[0 * kBlockM + r], l0 = xch[1 * kBlockM + r];
      const float m1 = xch[2 * kBlockM + r], l1 = xch[3 * kBlockM + r];
      const float m = fmaxf(m0, m1);
      const float a0 = (m0 == -INFINITY) ? 0.f : ex2_approx((m0 - m) * sl2);
      const float a1 = (m1 == -INFINITY) ? 0.f : ex2_approx((m1 - m) * sl2);
      const float l = l0 * a0 + l1 * a1;
      const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
      const float f0 = a0 * inv_l, f1 = a1 * inv_l;
      const bool in_range = row < args.N;
      T* orow = reinterpret_cast<T*>(args.o) +
                (static_cast<size_t>(bh) * static_cast<size_t>(args.N) + static_cast<size_t>(row)) * D;
      // Each warpgroup normalises and stores half of the head dimension.
#pragma unroll
      for (int c = g * (D / 2); c < (g + 1) * (D / 2); c += 32) {
        uint32_t u0[32];
        tmem_ld32_wait(tl + L::kColO + c, u0);
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(u0[i]) * f0;
        if (n_t1 > 0) {
          uint32_t u1[32];
          tmem_ld32_wait(tl + L::kColO + D + c, u1);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = fmaf(__uint_as_float(u1[i]), f1, o[i]);
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack2<T>(o[2 * i], o[2 * i + 1]);
        if (in_range) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
      if (g == 0 && in_range) {
        args.lse[static_cast<size_t>(bh) * static_cast<size_t>(args.N) + static_cast<size_t>(row)] =
            (l > 0.f && m != -INFINITY) ? fmaf(m, args.scale, logf(l)) : INFINITY;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static const EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      return nullptr;
    }
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// [heads, N, D] view of a contiguous [B, H, N, D] tensor; box = 128 bytes of D x `rows` rows.
// Rows past N (inside one head) are zero-filled by the TMA unit.
cudaError_t make_tmap(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes,
                      int D, int N, long long heads, int rows) {
  const EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return cudaErrorNotSupported;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(N),
                              static_cast<cuuint64_t>(heads)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * elem_bytes,
                                 static_cast<cuuint64_t>(N) * D * elem_bytes};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / elem_bytes),
                             static_cast<cuuint32_t>(rows), 1u};
  const cuuint32_t estride[3] = {1u, 1u, 1u};
  const CUresult r = enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estride,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

std::atomic<unsigned int> g_epoch_host{0};

template <typename T, int D, int BN, int STAGES, bool CAUSAL>
cudaError_t launch_impl(const LaunchArgs& a, cudaStream_t stream) {
  using L = Layout<D, BN, STAGES>;
  auto* kern = &fa_fwd_sm100_kernel<T, D, BN, STAGES, CAUSAL>;
  static std::atomic<unsigned long long> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if ((configured.load(std::memory_order_acquire) & bit) == 0) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemAlloc);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  const CUtensorMapDataType dt = std::is_same<T, __nv_bfloat16>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  alignas(64) CUtensorMap mq, mk, mv;
  const long long hq = static_cast<long long>(a.B) * a.H;
  const long long hkv = static_cast<long long>(a.B) * a.Hkv;
  if ((e = make_tmap(&mq, a.q, dt, 2, D, a.N, hq, kBlockM)) != cudaSuccess) return e;
  if ((e = make_tmap(&mk, a.k, dt, 2, D, a.N, hkv, BN)) != cudaSuccess) return e;
  if ((e = make_tmap(&mv, a.v, dt, 2, D, a.N, hkv, BN)) != cudaSuccess) return e;

  KArgs ka;
  ka.o = a.o;
  ka.lse = a.lse;
  ka.H = a.H;
  ka.Hkv = a.Hkv;
  ka.N = a.N;
  ka.n_q_tiles = (a.N + kBlockM - 1) / kBlockM;
  // K+V of all kv heads: keep head-interleaved order while it fits comfortably in L2.
  const double kv_bytes = 2.0 * static_cast<double>(hkv) * a.N * D * 2.0;
  ka.head_major = kv_bytes > 48.0 * 1024 * 1024 ? 1 : 0;
  ka.scale = a.scale;
  ka.scale_log2 = a.scale * 1.4426950408889634f;
  ka.timeout_ns = a.timeout_ns;
  unsigned int ep = g_epoch_host.fetch_add(1) + 1;
  if (ep == 0) ep = g_epoch_host.fetch_add(1) + 1;
  ka.epoch = ep;
  ka.skip_kv_tile = a.skip_kv_tile;
  const long long grid = hq * ka.n_q_tiles;
  if (grid <= 0 || grid > INT_MAX) return cudaErrorInvalidValue;
  kern<<<static_cast<unsigned int>(grid), kThreads, L::kSmemAlloc, stream>>>(mq, mk, mv, ka);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_d(const LaunchArgs& a, cudaStream_t s) {
  // STAGES per key-tile width: as deep as shared memory allows with one CTA per SM.
  constexpr int kStages128 = (D == 128) ? 3 : 4;
  switch (a.block_n) {
    case 128:
      return a.causal ? launch_impl<T, D, 128, kStages128, true>(a, s)
                      : launch_impl<T, D, 128, kStages128, false>(a, s);
    case 64:
      return a.causal ? launch_impl<T, D, 64, 4, true>(a, s) : launch_impl<T, D, 64, 4, false>(a, s);
    case 32:
      return a.causal ? launch_impl<T, D, 32, 4, true>(a, s) : launch_impl<T, D, 32, 4, false>(a, s);
    default:
      return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_t(const LaunchArgs& a, cudaStream_t s) {
  switch (a.D) {
    case 64:
      return launch_d<T, 64>(a, s);
    case 128:
      return launch_d<T, 128>(a, s);
    default:
      return cudaErrorNotSupported;
  }
}

}  // namespace

bool block_n_supported(int dtype, int D, int block_n) {
  if (D != 64 && D != 128) return false;
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return false;
  return block_n == 32 || block_n == 64 || block_n == 128;
}

int default_block_n(int /*dtype*/, int /*D*/, int /*N*/) { return 128; }

cudaError_t launch_forward(const LaunchArgs& a, cudaStream_t stream) {
  switch (a.dtype) {
    case FA_DTYPE_F16:
      return launch_t<__half>(a, stream);
    case FA_DTYPE_BF16:
      return launch_t<__nv_bfloat16>(a, stream);
    default:
      return cudaErrorNotSupported;
  }
}

cudaError_t read_and_clear_status(unsigned int* bits) {
  cudaError_t e = cudaDeviceSynchronize();
  unsigned int v = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
  if (e == cudaSuccess) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
  }
  if (bits != nullptr) *bits = v;
  if (e != cudaSuccess) return e;
  return v != 0 ? cudaErrorLaunchTimeout : cudaSuccess;
}

}  // namespace fa_sm100
