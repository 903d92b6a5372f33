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
// One CTA computes one 128-row query tile of one (batch, head).  Warp roles (256 threads):
//   warp 0      TMA producer: Q once, then K_j / V_j through a STAGES-deep shared-memory ring
//               (full/empty mbarrier pairs; K and V have separate slots so K_{j+STAGES} can land
//               while V_j is still being read).
//   warp 1      owns tensor memory (alloc/dealloc); lane 0 issues every tcgen05.mma:
//                 S_j  = Q K_j^T     (SS: both operands in smem, K-major, 128-byte swizzle)
//                 O   += P_j V_j     (TS: P from TMEM, V from smem as an MN-major operand)
//               in the order S_0, S_1, PV_0, S_2, PV_1, ... so S_{j+1} runs on the tensor core
//               while the softmax warps work on S_j.
//   warps 2-3   idle (they only join the final barrier).
//   warps 4-7   softmax warpgroup, one thread per query row (TMEM lane = row): tcgen05.ld of
//               the S row, masking, row max, exp2, P packed to 16 bit and written back to TMEM
//               with tcgen05.st, then the O correction when the running max moved.
//
// Tensor memory (columns; 128 lanes = 128 query rows): S double buffer [0, 2*BN),
// O accumulator [2*BN, 2*BN + D), P double buffer of BN/2 columns each after it.  P has its
// own buffers so the only tensor-core hazards are same-accumulator ones (PV_j after PV_{j-1}),
// which the hardware orders; everything else is ordered by tcgen05.commit -> mbarrier.
//
// O rescaling is lazy: the max used for the exponent (m_ref) only moves when the tile max
// exceeds it by more than 2^8 in exponent units, so P stays <= 256 (exact in fp16/bf16 range)
// and the O read-modify-write through TMEM is rare.  The final o = acc/l and lse use the same
// m_ref, so the result is the same function (FlashAttention-4's conditional rescaling).
//
// Every mbarrier wait is bounded (globaltimer); a wait that runs out sets a CTA-local abort flag,
// records a cause bit in g_status and the launch epoch in g_abort_epoch (so other CTAs of the
// same launch stop early), then the CTA drains its own TMA copies and MMAs, frees TMEM and exits.
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
constexpr int kThreads = 256;
constexpr int kSoftmaxThread0 = 128;  // warps 4..7
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
  static constexpr int kNumBars = 7 + 4 * STAGES;
  static constexpr int kMiscOff = kBarOff + 8 * kNumBars;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kSmemAlloc = kBytes + 1024;  // slack to align the base to 1024 bytes

  static constexpr int kColS0 = 0;
  static constexpr int kColS1 = BN;
  static constexpr int kColO = 2 * BN;
  static constexpr int kColP0 = 2 * BN + D;
  static constexpr int kColP1 = 2 * BN + D + BN / 2;
  static constexpr int kColsUsed = 3 * BN + D;
  static constexpr int kTmemCols = kColsUsed <= 32    ? 32
                                   : kColsUsed <= 64  ? 64
                                   : kColsUsed <= 128 ? 128
                                   : kColsUsed <= 256 ? 256
                                                      : 512;

  // Barrier indices.
  static constexpr int kBarQ = 0;
  static constexpr int kBarKFull = 1;                 // + stage
  static constexpr int kBarVFull = 1 + STAGES;        // + stage
  static constexpr int kBarKEmpty = 1 + 2 * STAGES;   // + stage
  static constexpr int kBarVEmpty = 1 + 3 * STAGES;   // + stage
  static constexpr int kBarSFull = 1 + 4 * STAGES;    // + buffer
  static constexpr int kBarPFull = 3 + 4 * STAGES;    // + buffer
  static constexpr int kBarODone = 5 + 4 * STAGES;
  static constexpr int kBarDrain = 6 + 4 * STAGES;

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
  const int n_tiles = (kv_end + BN - 1) / BN;

  if (threadIdx.x == 0) {
    mbar_init(bar(L::kBarQ), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar(L::kBarKFull + s), 1);
      mbar_init(bar(L::kBarVFull + s), 1);
      mbar_init(bar(L::kBarKEmpty + s), 1);
      mbar_init(bar(L::kBarVEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(L::kBarSFull + b), 1);
      mbar_init(bar(L::kBarPFull + b), kBlockM);
    }
    mbar_init(bar(L::kBarODone), 1);
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
      bool ok = wait_bounded(bar(L::kBarQ), 0u, w, kStQFull);
      auto issue_s = [&](int j) -> bool {
        const int s = j % STAGES;
        if (!wait_bounded(bar(L::kBarKFull + s), static_cast<uint32_t>(j / STAGES) & 1u, w,
                          kStKFull)) {
          return false;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + ((j & 1) ? L::kColS1 : L::kColS0);
        const uint32_t kb = sbase + L::kKOff + s * L::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t q_off = (kk / 4) * L::kQChunkBytes + (kk % 4) * 32;
          const uint32_t k_off = (kk / 4) * L::kKVChunkBytes + (kk % 4) * 32;
          umma_ss(d_tmem, sdesc_sw128(sbase + L::kQOff + q_off, 16, 1024),
                  sdesc_sw128(kb + k_off, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar(L::kBarSFull + (j & 1)));
        umma_commit(bar(L::kBarKEmpty + s));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles) {
          ok = issue_s(j + 1);
          if (!ok) break;
        }
        ok = wait_bounded(bar(L::kBarPFull + (j & 1)), static_cast<uint32_t>(j >> 1) & 1u, w,
                          kStPFull);
        if (!ok) break;
        const int s = j % STAGES;
        ok = wait_bounded(bar(L::kBarVFull + s), static_cast<uint32_t>(j / STAGES) & 1u, w,
                          kStVFull);
        if (!ok) break;
        tc_fence_after();
        const uint32_t vb = sbase + L::kVOff + s * L::kKVBytes;
        const uint32_t pa = tmem + ((j & 1) ? L::kColP1 : L::kColP0);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          umma_ts(tmem + L::kColO, pa + kk * 8, sdesc_sw128(vb + kk * 16 * 128, L::kKVChunkBytes, 1024),
                  kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(bar(L::kBarODone));
        umma_commit(bar(L::kBarVEmpty + s));
      }
      // Exit path: all MMAs this thread issued must be complete before TMEM is freed.
      umma_commit(bar(L::kBarDrain));
      wait_drain(bar(L::kBarDrain), 0u, args.timeout_ns);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax warpgroup
    const int r = static_cast<int>(threadIdx.x) - kSoftmaxThread0;  // row within the tile
    const int row = q0 + r;
    const uint32_t tl = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float sl2 = args.scale_log2;
    constexpr bool kRoundedNorm = std::is_same<T, __nv_bfloat16>::value;
    float m_ref = -INFINITY;  // max used in the exponents (raw score units)
    float l_sum = 0.f;        // running sum of the fp32 weights (-> lse)
    float lq_sum = 0.f;       // running sum of the rounded weights (bf16: -> 1/l of O)
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarSFull + (j & 1)),
                                                static_cast<uint32_t>(j >> 1) & 1u, w, kStSFull));
      if (!ok) break;
      tc_fence_after();
      float s[BN];
      const uint32_t scol = (j & 1) ? L::kColS1 : L::kColS0;
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t u[32];
        tmem_ld32_wait(tl + scol + c * 32, u);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(u[i]);
      }
      const int kv0 = j * BN;
      if ((CAUSAL && kv0 + BN - 1 > q0) || kv0 + BN > args.N) {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const int kv = kv0 + c;
          if (kv >= args.N || (CAUSAL && kv > row)) s[c] = -INFINITY;
        }
      }
      float tmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; ++c) tmax = fmaxf(tmax, s[c]);
      const float m_new = fmaxf(m_ref, tmax);
      const bool resc = (m_ref == -INFINITY) ? (m_new != -INFINITY)
                                             : ((m_new - m_ref) * sl2 > kRescaleThreshold);
      const float m_use = resc ? m_new : m_ref;
      const float alpha =
          resc ? ((m_ref == -INFINITY) ? 0.f : ex2_approx((m_ref - m_use) * sl2)) : 1.f;
      const float mc = (m_use == -INFINITY) ? 0.f : m_use * sl2;
      float rs = 0.f;   // sum of the fp32 weights: the logsumexp uses this one
      float rsq = 0.f;  // bf16 only: sum of the rounded weights, the normaliser of O
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN / 2; ++c) {
        const float p0 = ex2_approx(fmaf(s[2 * c], sl2, -mc));
        const float p1 = ex2_approx(fmaf(s[2 * c + 1], sl2, -mc));
        pk[c] = pack2<T>(p0, p1);
        rs += p0 + p1;
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          // bf16 keeps 8 significant bits: O is normalised by the sum of the ROUNDED weights
          // the tensor core multiplies, so o stays a convex combination of V rows and the
          // common-mode part of the rounding error cancels (rows with few keys).
          rsq += __uint_as_float(pk[c] << 16) + __uint_as_float(pk[c] & 0xFFFF0000u);
        }
      }
      const uint32_t pcol = (j & 1) ? L::kColP1 : L::kColP0;
#pragma unroll
      for (int c = 0; c < BN / 2; c += 16) tmem_st16(tl + pcol + c, &pk[c]);
      tmem_st_wait();
      l_sum = l_sum * alpha + rs;
      if constexpr (kRoundedNorm) lq_sum = lq_sum * alpha + rsq;
      m_ref = m_use;
      if (j > 0) {
        // PV_{j-1} must be complete before O may be touched (and, for phase bookkeeping, it is
        // waited for on every tile: it finished long ago in the common case).
        ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarODone),
                                                  static_cast<uint32_t>(j - 1) & 1u, w, kStODone));
        if (!ok) break;
        if (__any_sync(0xffffffffu, resc)) {
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D; c += 32) {
            uint32_t u[32];
            tmem_ld32_wait(tl + L::kColO + c, u);
#pragma unroll
            for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
            tmem_st32(tl + L::kColO + c, u);
          }
          tmem_st_wait();
        }
      }
      tc_fence_before();
      mbar_arrive(bar(L::kBarPFull + (j & 1)));
    }
    if (ok) {
      ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarODone),
                                                static_cast<uint32_t>(n_tiles - 1) & 1u, w,
                                                kStODone));
    }
    if (ok) {
      tc_fence_after();
      const float l_norm = kRoundedNorm ? lq_sum : l_sum;
      const float inv_l = (l_norm > 0.f) ? 1.f / l_norm : 0.f;
      const bool in_range = row < args.N;
      T* orow = reinterpret_cast<T*>(args.o) +
                (static_cast<size_t>(bh) * static_cast<size_t>(args.N) + static_cast<size_t>(row)) * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t u[32];
        tmem_ld32_wait(tl + L::kColO + c, u);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          pk[i] = pack2<T>(__uint_as_float(u[2 * i]) * inv_l, __uint_as_float(u[2 * i + 1]) * inv_l);
        }
        if (in_range) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
      if (in_range) {
        args.lse[static_cast<size_t>(bh) * static_cast<size_t>(args.N) + static_cast<size_t>(row)] =
            (l_sum > 0.f && m_ref != -INFINITY) ? fmaf(m_ref, args.scale, logf(l_sum)) : INFINITY;
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
  constexpr int kStages128 = (D == 128) ? 2 : 4;
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
