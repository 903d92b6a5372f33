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
// Two kernels live in this translation unit (one set of device status words):
//   * fa_fwd_lookahead_kernel (fa_fwd_lookahead.cuh): fp16/bf16 with 128-key rounds split 64/64
//     between the softmax warpgroups, P and Q in their own tensor-memory columns, S one round
//     ahead -- selected by block_n = 64, the default for D = 128;
//   * fa_fwd_sm100_kernel (below): P written over S, whole key tiles alternating between the
//     warpgroups -- block_n = 128 (the default for D = 64) and 32, and every fp32 (tf32) launch.
// Both walk the same persistent item order (fa_kernel_common.cuh).
//
// Persistent CTAs, one per SM (each needs all 512 TMEM columns and ~220 KB of shared memory), each
// walking a fixed list of work items -- one 128-row query tile of one (batch, head) -- in a
// balanced order (see decode_item).  Warp roles (384 threads):
//   warp 0      TMA producer: each item's Q tile (after the previous item's S MMAs released the
//               buffer) and the K tiles through a KST-deep ring (full/empty mbarrier pairs).
//   warp 1      owns tensor memory (alloc/dealloc); lane 0 issues every tcgen05.mma.
//   warp 2      TMA producer of the V tiles through a VST-deep ring.
//   warp 3      idle (it only joins the final barrier).
//   warps 4-7   softmax warpgroup 0: key tiles j = 0, 2, 4, ... of each item
//   warps 8-11  softmax warpgroup 1: key tiles j = 1, 3, 5, ... of each item
// Barrier phases run on across items.  The next item's first S MMAs overlap the current item's
// merge/store epilogue; its first PV (which overwrites O) waits for the o_free barrier that the
// 256 softmax threads arrive on once they have read O_0 and O_1.
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

// O rescaling is lazy for fp16 and tf32: the max used for the exponent (m_ref) only moves when the
// tile max exceeds it by more than 2^8 in exponent units, so P stays <= 256 (in range) and the O
// read-modify-write through TMEM is rare.  The final o = acc/l and lse use the same m_ref, so the
// result is the same function (FlashAttention-4's conditional rescaling).  bf16 rescales whenever
// the max grows: with 8 significant bits, a weight above 1 that dominates its row would carry
// its rounding error straight into O.
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

#include "fa_fwd_lookahead.cuh"
#include "fa_kernel_common.cuh"
#include "fa_launch.h"
#include "fa_sm100.h"
#include "sm100_ptx.cuh"

namespace fa_sm100 {
namespace {

template <int EB, int D, int BN, int KST, int VST>
struct Layout {
  static constexpr int kEB = EB;                 // bytes per element (2: fp16/bf16, 4: fp32)
  static constexpr int kSwElems = 128 / kEB;     // elements per 128-byte swizzle row
  static constexpr int kDChunks = D / kSwElems;  // 128-byte column chunks along D
  static constexpr int kQChunkBytes = kBlockM * 128;
  static constexpr int kKVChunkBytes = BN * 128;
  static constexpr int kQBytes = kBlockM * D * kEB;
  static constexpr int kKVBytes = BN * D * kEB;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + KST * kKVBytes;
  // 16-bit: O staging for the epilogue's TMA store (128-byte-swizzled 128-row chunks of 64
  // columns, like the Q tile), with the merge's (m, l) exchange at its start -- it is read before
  // O is staged.  fp32 stores O directly and keeps only the exchange.
  static constexpr int kOStOff = kVOff + VST * kKVBytes;
  static constexpr int kXchBytes = 2 * 2 * kBlockM * 4 + 16;
  static constexpr int kOStBytes = EB == 2 ? kBlockM * D * 2 : kXchBytes;
  static constexpr int kXchOff = kOStOff;  // merge exchange: m, l per row and group
  static constexpr int kBarOff = kOStOff + kOStBytes;
  static constexpr int kNumBars = 10 + 2 * KST + 2 * VST;
  static constexpr int kMiscOff = kBarOff + 8 * kNumBars;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kSmemAlloc = kBytes + 1024;  // slack to align the base to 1024 bytes

  // Tensor memory columns.
  static constexpr int kColS = 0;       // + g * BN
  static constexpr int kColO = 2 * BN;  // + g * D
  static constexpr int kColsUsed = 2 * BN + 2 * D;
  static constexpr int kTmemCols = kColsUsed <= 32    ? 32
                                   : kColsUsed <= 64  ? 64
                                   : kColsUsed <= 128 ? 128
                                   : kColsUsed <= 256 ? 256
                                                      : 512;

  // Barrier indices.
  static constexpr int kBarQFull = 0;
  static constexpr int kBarQEmpty = 1;
  static constexpr int kBarSFull = 2;   // + group
  static constexpr int kBarPFull = 4;   // + group
  static constexpr int kBarPVDone = 6;  // + group
  static constexpr int kBarOFree = 8;
  static constexpr int kBarDrain = 9;
  static constexpr int kBarKFull = 10;                   // + stage
  static constexpr int kBarKEmpty = 10 + KST;            // + stage
  static constexpr int kBarVFull = 10 + 2 * KST;         // + stage
  static constexpr int kBarVEmpty = 10 + 2 * KST + VST;  // + stage

  // tcgen05.mma steps: 32 bytes of K per instruction (16 fp16/bf16 or 8 tf32 elements).
  static constexpr int kSSteps = D * EB / 32;     // S = Q K^T: K dimension = D
  static constexpr int kPVSteps = BN * EB / 32;   // O += P V: K dimension = BN keys
  static constexpr int kPVStepBytes = (32 / EB) * 128;  // V rows consumed per step x 128 B

  static_assert(D % kSwElems == 0, "D must be a multiple of the swizzle width");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 128, "BN must be 32, 64 or 128");
  static_assert(kColsUsed <= 512, "tensor memory overflow");
  static_assert(kSmemAlloc <= 232448, "shared memory overflow");
};


template <typename T, int D, int BN, int KST, int VST, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_o, const KArgs args) {
  using L = Layout<static_cast<int>(sizeof(T)), D, BN, KST, VST>;
  constexpr bool kTf32 = std::is_same<T, float>::value;
  constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : (kTf32 ? 2u : 0u);
  // Rescale threshold (log2 units).  fp16 P and tf32 P keep 11 significant bits, so weights up to
  // 2^8 (lazy rescaling) cost nothing; bf16 keeps 8, and a row dominated by one key must keep its
  // largest weight exactly 1 (rescale whenever the running max grows), or that weight's rounding
  // alone moves O past the 8e-3 gate.
  constexpr float kResc = std::is_same<T, __nv_bfloat16>::value ? 0.0f : kRescaleThreshold;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  auto bar = [sbase](int i) -> uint32_t { return sbase + L::kBarOff + 8u * i; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x);
  const int cta = static_cast<int>(blockIdx.x);

  int pre_k = 0;  // K tiles of the first item issued in the prologue (thread 0 only)
  if (threadIdx.x == 0) {
#ifdef FA_TRACE
    if (blockIdx.x < kTraceCtas) g_trace_t0[blockIdx.x] = clock64();
#endif
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    mbar_init(bar(L::kBarQFull), 1);
    mbar_init(bar(L::kBarQEmpty), 1);
    for (int g = 0; g < 2; ++g) {
      mbar_init(bar(L::kBarSFull + g), 1);
      mbar_init(bar(L::kBarPFull + g), kBlockM);

      mbar_init(bar(L::kBarPVDone + g), 1);
    }
    mbar_init(bar(L::kBarOFree), 2 * kBlockM);
    mbar_init(bar(L::kBarDrain), 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(bar(L::kBarKFull + s), 1);
      mbar_init(bar(L::kBarKEmpty + s), 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(bar(L::kBarVFull + s), 1);
      mbar_init(bar(L::kBarVEmpty + s), 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
    // Thread 0 is also the Q/K producer: the first item's Q and first K tiles go out now, ahead of
    // the tensor-memory allocation and the CTA barrier (at a cold start they come from DRAM, and
    // the first S waits for them); the producer loop skips them.
    const Item it0 = decode_item<CAUSAL>(item_index(0, G, cta), args);
    const Heads hd0 = split_heads(it0.bh, args);
    const int kv_end0 = CAUSAL ? min(args.N, it0.q_tile * kBlockM + kBlockM) : args.N;
    mbar_arrive_expect_tx(bar(L::kBarQFull), L::kQBytes);
#pragma unroll
    for (int c = 0; c < L::kDChunks; ++c) {
      tma_load_view(sbase + L::kQOff + c * L::kQChunkBytes, &tm_q, c * L::kSwElems,
                    it0.q_tile * kBlockM, hd0.h, hd0.b, args.q_pos, bar(L::kBarQFull));
    }
    pre_k = min(KST, (kv_end0 + BN - 1) / BN);
    for (int j = 0; j < pre_k; ++j) {
      if (j == args.skip_kv_tile) continue;
      mbar_arrive_expect_tx(bar(L::kBarKFull + j), L::kKVBytes);
#pragma unroll
      for (int c = 0; c < L::kDChunks; ++c) {
        tma_load_view(sbase + L::kKOff + j * L::kKVBytes + c * L::kKVChunkBytes, &tm_k,
                      c * L::kSwElems, j * BN, hd0.hk, hd0.b, args.k_pos, bar(L::kBarKFull + j));
      }
    }
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

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------------ TMA producers
    // warp 0: Q of every item and the K ring; warp 2: the V ring.  Each walks the CTA's items.
    if (lane == 0) {
      const bool is_k = (warp == 0);
      constexpr int kStMax = KST > VST ? KST : VST;
      const int nst = is_k ? KST : VST;
      const int bar_full = is_k ? L::kBarKFull : L::kBarVFull;
      const int bar_empty = is_k ? L::kBarKEmpty : L::kBarVEmpty;
      const uint32_t ring = sbase + (is_k ? L::kKOff : L::kVOff);
      const CUtensorMap* tm = is_k ? &tm_k : &tm_v;
      if (!is_k) tma_prefetch_desc(tm);
      int count = 0;        // tiles this producer has issued, over all items
      int items_done = 0;   // items whose Q this producer loaded (warp 0)
      unsigned skipped = 0;  // bit (count % 32): that tile's copy was skipped (fault injection)
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int i = item_index(r, G, cta);
        if (i >= args.n_items) break;
        const Item item = decode_item<CAUSAL>(i, args);
        const int q0 = item.q_tile * kBlockM;
        const Heads hd = split_heads(item.bh, args);
        const int kv_end = CAUSAL ? min(args.N, q0 + kBlockM) : args.N;
        const int n_tiles = (kv_end + BN - 1) / BN;
        if (is_k) {
          // The previous item's S MMAs must be done with the Q buffer.
          if (items_done > 0 &&
              !(ok = wait_bounded(bar(L::kBarQEmpty), static_cast<uint32_t>(items_done - 1) & 1u,
                                  w, kStKVEmpty))) {
            break;
          }
          if (items_done > 0) {  // the first item's Q went out in the prologue
            mbar_arrive_expect_tx(bar(L::kBarQFull), L::kQBytes);
#pragma unroll
            for (int c = 0; c < L::kDChunks; ++c) {
              tma_load_view(sbase + L::kQOff + c * L::kQChunkBytes, &tm_q, c * L::kSwElems, q0,
                            hd.h, hd.b, args.q_pos, bar(L::kBarQFull));
            }
          }
          ++items_done;
        }
        for (int j = 0; j < n_tiles; ++j, ++count) {
          const int s = count % nst;
          const uint32_t ph = static_cast<uint32_t>(count / nst) & 1u;
          if (count >= nst && !(ok = wait_bounded(bar(bar_empty + s), ph ^ 1u, w, kStKVEmpty))) {
            break;
          }
          if (is_k && j == args.skip_kv_tile) {
            skipped |= 1u << (count & 31);
            continue;
          }
          skipped &= ~(1u << (count & 31));
          if (is_k && r == 0 && j < pre_k) continue;  // issued in the prologue
          mbar_arrive_expect_tx(bar(bar_full + s), L::kKVBytes);
#pragma unroll
          for (int c = 0; c < L::kDChunks; ++c) {
            tma_load_view(ring + s * L::kKVBytes + c * L::kKVChunkBytes, tm, c * L::kSwElems,
                          j * BN, hd.hk, hd.b, is_k ? args.k_pos : args.v_pos, bar(bar_full + s));
          }
        }
      }
      (void)kStMax;
      // Exit path: every copy this thread started must have landed before the CTA may exit.
      if (is_k && items_done > 0) {
        wait_drain(bar(L::kBarQFull), static_cast<uint32_t>(items_done - 1) & 1u, args.timeout_ns);
      }
      for (int c = (count > nst ? count - nst : 0); c < count; ++c) {
        if (!((skipped >> (c & 31)) & 1u)) {
          wait_drain(bar(bar_full + c % nst), static_cast<uint32_t>(c / nst) & 1u, args.timeout_ns);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescS = idesc_mma(kFmt, kBlockM, BN, false);
      constexpr uint32_t kIdescPV = idesc_mma(kFmt, kBlockM, D, true);
      // Descriptor bases; an offset inside a tile is added to the start-address field (the sum
      // stays below 2^14 in 16-byte units for any shared-memory address, so it cannot carry).
      const uint64_t q_desc0 = sdesc_sw128(sbase + L::kQOff, 16, 1024);
      const uint64_t k_desc0 = sdesc_sw128(sbase + L::kKOff, 16, 1024);
      // V is the MN-major B operand (D contiguous).  16-bit: 128-byte swizzle, 8-row K groups;
      // tf32: 128-byte swizzle with 32-byte atoms, 4-row K groups.
      const uint64_t v_desc0 = kTf32 ? sdesc_sw128_atom32(sbase + L::kVOff, L::kKVChunkBytes, 512)
                                     : sdesc_sw128(sbase + L::kVOff, L::kKVChunkBytes, 1024);
      int kc = 0, vc = 0;   // K / V tiles consumed, over all items
      int pc[2] = {0, 0};   // P tiles consumed per group, over all items
      int it = 0;           // items processed
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int i = item_index(r, G, cta);
        if (i >= args.n_items) break;
        const Item item = decode_item<CAUSAL>(i, args);
        const int q0 = item.q_tile * kBlockM;
        const int kv_end = CAUSAL ? min(args.N, q0 + kBlockM) : args.N;
        const int n_tiles = (kv_end + BN - 1) / BN;
        const int n_t0 = (n_tiles + 1) / 2, n_t1 = n_tiles / 2;
        const bool comp = std::is_same<T, __nv_bfloat16>::value && CAUSAL && item.q_tile == 0;
        int s_issued = 0;  // S MMAs of this item
        // S_g = Q K_j^T into S_g; the commit after the item's last S releases the Q buffer.
        auto issue_s = [&](int g, int t) -> bool {
          const int s = kc % KST;
          if (!wait_bounded(bar(L::kBarKFull + s), static_cast<uint32_t>(kc / KST) & 1u, w,
                            kStKFull)) {
            return false;
          }
          tc_fence_after();
          FA_TRACE_EV(it == 0, 0, g, t);
          const uint32_t d_tmem = tmem + L::kColS + g * BN;
          const uint64_t k_desc = k_desc0 + static_cast<uint64_t>((s * L::kKVBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < L::kSSteps; ++kk) {
            const uint32_t q_off = (kk / 4) * L::kQChunkBytes + (kk % 4) * 32;
            const uint32_t k_off = (kk / 4) * L::kKVChunkBytes + (kk % 4) * 32;
            if constexpr (kTf32) {
              umma_ss_tf32(d_tmem, q_desc0 + (q_off >> 4), k_desc + (k_off >> 4), kIdescS,
                           kk > 0 ? 1u : 0u);
            } else {
              umma_ss(d_tmem, q_desc0 + (q_off >> 4), k_desc + (k_off >> 4), kIdescS,
                      kk > 0 ? 1u : 0u);
            }
          }
          umma_commit(bar(L::kBarSFull + g));
          umma_commit(bar(L::kBarKEmpty + s));
          ++kc;
          if (++s_issued == n_tiles) umma_commit(bar(L::kBarQEmpty));
          return true;
        };
        // O_g += P_g V_j (twice with `comp`: P_hi then P_lo from the second half of S_g).
        auto issue_pv = [&](int g, int t, bool last) -> bool {
          const int s = vc % VST;
          if (!wait_bounded(bar(L::kBarPFull + g), static_cast<uint32_t>(pc[g]) & 1u, w,
                            kStPFull)) {
            return false;
          }
          ++pc[g];
          if (!wait_bounded(bar(L::kBarVFull + s), static_cast<uint32_t>(vc / VST) & 1u, w,
                            kStVFull)) {
            return false;
          }
          tc_fence_after();
          FA_TRACE_EV(it == 0, 1, g, t);
          const uint64_t v_desc = v_desc0 + static_cast<uint64_t>((s * L::kKVBytes) >> 4);
          const uint32_t pa = tmem + L::kColS + g * BN;
          const uint32_t o_tmem = tmem + L::kColO + g * D;
          // Each step reads 8 TMEM columns of P (16 packed 16-bit weights or 8 fp32 ones).
#pragma unroll
          for (int kk = 0; kk < L::kPVSteps; ++kk) {
            const uint64_t vd = v_desc + ((kk * L::kPVStepBytes) >> 4);
            if constexpr (kTf32) {
              umma_ts_tf32(o_tmem, pa + kk * 8, vd, kIdescPV, (t > 0 || kk > 0) ? 1u : 0u);
            } else {
              umma_ts(o_tmem, pa + kk * 8, vd, kIdescPV, (t > 0 || kk > 0) ? 1u : 0u);
            }
          }
          if constexpr (!kTf32) {
            if (comp) {
#pragma unroll
              for (int kk = 0; kk < L::kPVSteps; ++kk) {
                umma_ts(o_tmem, pa + BN / 2 + kk * 8, v_desc + ((kk * L::kPVStepBytes) >> 4),
                        kIdescPV, 1u);
              }
            }
          }
          if (last) umma_commit(bar(L::kBarPVDone + g));
          umma_commit(bar(L::kBarVEmpty + s));
          ++vc;
          return true;
        };
        // Order: S_0(0), S_1(0), then per round PV_0(t), S_0(t+1), PV_1(t), S_1(t+1): the tensor
        // core works for one group while the other runs its softmax.  S_g(t+1) overwrites the
        // TMEM columns PV_g(t) reads right after it; tcgen05.mma instructions issued by one
        // thread execute in issue order, so the reads come first (FlashAttention-4's forward
        // schedules the same pair the same way).  The first S of an item may overlap the
        // previous item's epilogue (S and O are distinct columns); its first PV (which
        // overwrites O_g) waits until that epilogue has read both O_g.
        if (!(ok = wait_bounded(bar(L::kBarQFull), static_cast<uint32_t>(it) & 1u, w, kStQFull))) {
          break;
        }
        if (!(ok = issue_s(0, 0))) break;
        if (n_t1 > 0 && !(ok = issue_s(1, 0))) break;
        if (it > 0 && !(ok = wait_bounded(bar(L::kBarOFree), static_cast<uint32_t>(it - 1) & 1u,
                                          w, kStODone))) {
          break;
        }
        for (int t = 0; ok && t < n_t0; ++t) {
          if (!(ok = issue_pv(0, t, t + 1 == n_t0))) break;
          if (t + 1 < n_t0 && !(ok = issue_s(0, t + 1))) break;
          if (t < n_t1) {
            if (!(ok = issue_pv(1, t, t + 1 == n_t1))) break;
            if (t + 1 < n_t1 && !(ok = issue_s(1, t + 1))) break;
          }
        }
        ++it;
      }
      // Exit path: all MMAs this thread issued must be complete before TMEM is freed.
      umma_commit(bar(L::kBarDrain));
      wait_drain(bar(L::kBarDrain), 0u, args.timeout_ns);
    }
    __syncwarp();
  } else if (warp >= kSoftmaxWarp0) {
    // ------------------------------------------------------------------ softmax warpgroups
    const int g = (warp - kSoftmaxWarp0) >> 2;  // 0: even key tiles, 1: odd key tiles
    const int r = (warp & 3) * 32 + lane;       // row within the tile == TMEM lane
    const uint32_t tl = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_col = L::kColS + g * BN;
    const uint32_t o_col = L::kColO + g * D;
    const float sl2 = args.scale_log2;
    float* xch = reinterpret_cast<float*>(smem + L::kXchOff);
    volatile int* xch_ctl = reinterpret_cast<volatile int*>(smem + L::kXchOff + 2 * 2 * kBlockM * 4);
    // The thread that issues O's TMA stores (16-bit; fp32 writes O directly).
    const bool o_issuer = !kTf32 && g == 0 && warp == kSoftmaxWarp0 && lane == 0;
    if (o_issuer) tma_prefetch_desc(&tm_o);
    int sc = 0;   // S tiles consumed by this group, over all items
    int pvc = 0;  // item-final PV completions consumed by this group
    for (int rnd = 0;; ++rnd) {
      const int i = item_index(rnd, G, cta);
      if (i >= args.n_items) break;
      const Item item = decode_item<CAUSAL>(i, args);
      (void)FA_DCHECK(item.bh < args.n_bh && item.q_tile >= 0 && item.q_tile < args.n_q_tiles);
      const int q0 = item.q_tile * kBlockM;
      const int row = q0 + r;
      const int kv_end = CAUSAL ? min(args.N, q0 + kBlockM) : args.N;
      const int n_tiles = (kv_end + BN - 1) / BN;
      const int n_t1 = n_tiles / 2;
      const int n_t = (g == 0) ? (n_tiles + 1) / 2 : n_t1;
      const bool comp = std::is_same<T, __nv_bfloat16>::value && CAUSAL && item.q_tile == 0;
      float m_ref = -INFINITY;  // max used in the exponents (raw score units)
      float l_sum = 0.f;        // running sum of the fp32 weights
      bool ok = true;
      for (int t = 0; t < n_t; ++t) {
        const int j = 2 * t + g;
        ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarSFull + g),
                                                  static_cast<uint32_t>(sc) & 1u, w, kStSFull));
        if (!ok) break;
        ++sc;
        tc_fence_after();
        FA_TRACE_EV(rnd == 0 && r == 0, 2, g, t);
        float s[BN];
        if (FA_DCHECK(s_col + BN <= L::kTmemCols)) load_s_row<BN>(tl + s_col, s);
        FA_TRACE_EV(rnd == 0 && r == 0, 4, g, t);
        const int kv0 = j * BN;
        if ((CAUSAL && kv0 + BN - 1 > q0) || kv0 + BN > args.N) {
          // Key kv0 + c is visible to this row iff c <= lim (top-left causal, inside N).
          const int lim = (CAUSAL ? min(row, args.N - 1) : args.N - 1) - kv0;
#pragma unroll
          for (int c = 0; c < BN; ++c) s[c] = (c > lim) ? -INFINITY : s[c];
        }
        const float m_new = fmaxf(m_ref, row_max<BN>(s));
        const bool resc = (m_ref == -INFINITY) ? (m_new != -INFINITY)
                                               : ((m_new - m_ref) * sl2 > kResc);
        const float m_use = resc ? m_new : m_ref;
        const float alpha =
            resc ? ((m_ref == -INFINITY) ? 0.f : ex2_approx((m_ref - m_use) * sl2)) : 1.f;
        const float mc = (m_use == -INFINITY) ? 0.f : m_use * sl2;
        FA_TRACE_EV(rnd == 0 && r == 0, 5, g, t);
        // P_g over the first half of S_g (all of S_g's row is in registers by now).
        float rs;
        if constexpr (kTf32) {
          rs = exp_store_f32<BN>(s, sl2, mc, tl + s_col);
        } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          rs = comp ? exp_pack_store<T, BN, 0, BN / 2, true>(s, sl2, mc, tl + s_col)
                    : exp_pack_store<T, BN, 0, BN / 2, false>(s, sl2, mc, tl + s_col);
        } else {
          rs = exp_pack_store<T, BN, 0, BN / 2, false>(s, sl2, mc, tl + s_col);
        }
        tmem_st_wait();
        l_sum = l_sum * alpha + rs;
        m_ref = m_use;
        // O_g correction.  S_g(t) completing implies PV_g(t-1) completed (the commit of S_g(t)
        // covers every MMA issued before it), and PV_g(t) waits for our arrival below.
        if (t > 0 && __any_sync(0xffffffffu, resc) && FA_DCHECK(o_col + D <= L::kTmemCols)) {
#pragma unroll
          for (int c = 0; c < D; c += 32) {
            uint32_t u[32];
            tmem_ld32_wait(tl + o_col + c, u);
#pragma unroll
            for (int k2 = 0; k2 < 32; ++k2) u[k2] = __float_as_uint(__uint_as_float(u[k2]) * alpha);
            tmem_st32(tl + o_col + c, u);
          }
          tmem_st_wait();
        }
        tc_fence_before();
        FA_TRACE_EV(rnd == 0 && r == 0, 3, g, t);
        mbar_arrive(bar(L::kBarPFull + g));
      }
      // ---- merge the two partials; O / LSE (16-bit: O staged and written by TMA) ----------
      if (ok && n_t > 0) {  // committed once per item, after the group's last PV
        ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarPVDone + g),
                                                  static_cast<uint32_t>(pvc) & 1u, w, kStODone));
        ++pvc;
      }
      // The previous item's O store must have read the staging buffer (the exchange lives there).
      if (o_issuer) bulk_wait_read();
      tc_fence_before();
      // Both groups reach both named barriers once per item, on the abort path too; whether to
      // merge and go on is decided by one thread and read by all after the second barrier.
      named_barrier_sync(kMergeBarrier, 2 * kBlockM);
      xch[(g * 2 + 0) * kBlockM + r] = m_ref;
      xch[(g * 2 + 1) * kBlockM + r] = l_sum;
      if (g == 0 && r == 0) *xch_ctl = *abort_flag;
      named_barrier_sync(kMergeBarrier, 2 * kBlockM);
      if (*xch_ctl != 0) break;
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
      if constexpr (!kTf32) {
        // Every thread has read the exchange before O overwrites it.
        named_barrier_sync(kMergeBarrier, 2 * kBlockM);
      }
      T* orow = out_row<T>(args, item.bh, row);
      // Each group normalises half of the head dimension: fp32 straight to global memory; 16-bit
      // into the staging buffer (row r of 64-column chunk c at kOStOff + c*16 KB + r*128 B, 16-byte
      // units XOR-swizzled by r % 8, the layout of the O tensor map's 128-byte swizzle).
#pragma unroll
      for (int c = g * (D / 2); c < (g + 1) * (D / 2); c += 32) {
        uint32_t u0[32];
        tmem_ld32_wait(tl + L::kColO + c, u0);
        float o[32];
#pragma unroll
        for (int k2 = 0; k2 < 32; ++k2) o[k2] = __uint_as_float(u0[k2]) * f0;
        if (n_t1 > 0) {
          uint32_t u1[32];
          tmem_ld32_wait(tl + L::kColO + D + c, u1);
#pragma unroll
          for (int k2 = 0; k2 < 32; ++k2) o[k2] = fmaf(__uint_as_float(u1[k2]), f1, o[k2]);
        }
        if constexpr (kTf32) {
          if (in_range && FA_DCHECK(item.bh < args.n_bh && c + 32 <= D)) {
            float4* dst = reinterpret_cast<float4*>(orow + c);
#pragma unroll
            for (int k2 = 0; k2 < 8; ++k2) {
              dst[k2] = make_float4(o[4 * k2], o[4 * k2 + 1], o[4 * k2 + 2], o[4 * k2 + 3]);
            }
          }
        } else {
          uint32_t pk[16];
#pragma unroll
          for (int k2 = 0; k2 < 16; ++k2) pk[k2] = pack2<T>(o[2 * k2], o[2 * k2 + 1]);
          uint8_t* rowp = smem + L::kOStOff + (c / 64) * L::kQChunkBytes + r * 128;
          if (!FA_DCHECK((c / 64) * L::kQChunkBytes + r * 128 + 128 <= L::kOStBytes)) continue;
#pragma unroll
          for (int k2 = 0; k2 < 4; ++k2) {
            const int unit = (c % 64) / 8 + k2;
            *reinterpret_cast<uint4*>(rowp + ((unit ^ (r & 7)) << 4)) =
                make_uint4(pk[4 * k2], pk[4 * k2 + 1], pk[4 * k2 + 2], pk[4 * k2 + 3]);
          }
        }
      }
      // O_0 and O_1 have been read: the next item's first PVs may overwrite them.
      tc_fence_before();
      mbar_arrive(bar(L::kBarOFree));
      if (g == 0 && in_range && FA_DCHECK(item.bh < args.n_bh)) {
        args.lse[static_cast<size_t>(item.bh) * static_cast<size_t>(args.N) + static_cast<size_t>(row)] =
            (l > 0.f && m != -INFINITY) ? fmaf(m, args.scale, logf(l)) : INFINITY;
      }
      if constexpr (!kTf32) {
        // The staged tile goes out in one TMA store per 64-column chunk (rows past N are
        // clipped); it overlaps the next item.
        fence_proxy_async_smem();
        named_barrier_sync(kMergeBarrier, 2 * kBlockM);
        if (o_issuer) {
          const Heads hd = split_heads(item.bh, args);
#pragma unroll
          for (int c = 0; c < L::kDChunks; ++c) {
            tma_store_view(&tm_o, sbase + L::kOStOff + c * L::kQChunkBytes, c * 64, q0, hd.h, hd.b,
                           args.o_pos);
          }
          bulk_commit();
        }
      }
    }
    // The last O store must have completed before the CTA exits.
    if (o_issuer) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

// fp32 inputs would enter the tf32 tensor core with their low 13 mantissa bits dropped
// (truncation: a bias toward zero that shifts every score the same way).  The fp32 path first
// rounds q, k and v to tf32 (round to nearest, ties away) into the caller's workspace as
// contiguous [B, H, N, D] copies laid out [q | k | v], gathering from any (b, h, n) strides, so
// the products carry unbiased rounding errors.  HBM-bound: 16 bytes in and out per thread and
// step, grid-stride.
struct View4 {
  const float* p;
  long long sb, sh, sn;  // element strides; d contiguous
  int heads;
  size_t units;          // 16-byte units of the contiguous copy
};

__device__ __forceinline__ uint4 load_view_unit(const View4& v, size_t u, int N, int d4) {
  const size_t row = u / d4;  // (b * heads + h) * N + n
  const int c = static_cast<int>(u - row * d4);
  const size_t bh = row / N;
  const int n = static_cast<int>(row - bh * N);
  const size_t b = bh / v.heads;
  const int h = static_cast<int>(bh - b * v.heads);
  const float* src = v.p + b * v.sb + h * v.sh + n * v.sn + 4 * c;
  return *reinterpret_cast<const uint4*>(src);
}

__global__ void __launch_bounds__(256)
    fa_round_tf32_kernel(View4 q, View4 k, View4 v, int N, int d4, uint4* __restrict__ out) {
  const size_t n = q.units + k.units + v.units;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint4 x = i < q.units ? load_view_unit(q, i, N, d4)
                    : i < q.units + k.units ? load_view_unit(k, i - q.units, N, d4)
                                            : load_view_unit(v, i - q.units - k.units, N, d4);
    out[i] = make_uint4(f32_to_tf32(__uint_as_float(x.x)), f32_to_tf32(__uint_as_float(x.y)),
                        f32_to_tf32(__uint_as_float(x.z)), f32_to_tf32(__uint_as_float(x.w)));
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

// [b][h][n][d] view of q/k/v with element strides st = {b, h, n} (d contiguous) as a 4-D tensor
// map.  Dimension 0 is d (box = 128 bytes of it); dimensions 1-3 are n, h, b sorted by stride
// (the encoder's layout model has each stride include the previous one); `pos` returns, packed
// two bits each, the map dimension (0-2 among dims 1-3) holding n, h and b.  Rows past N are
// zero-filled by the TMA unit.
cudaError_t make_tmap(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes,
                      int D, int N, int heads, int B, int rows, const long long st[3],
                      CUtensorMapSwizzle swizzle, int* pos) {
  const EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return cudaErrorNotSupported;
  const long long stride[3] = {st[2], st[1], st[0]};  // n, h, b
  const long long size[3] = {N, heads, B};
  int order[3] = {0, 1, 2};
  for (int i = 1; i < 3; ++i) {  // stable insertion sort by stride
    for (int j = i; j > 0 && stride[order[j]] < stride[order[j - 1]]; --j) {
      const int t = order[j];
      order[j] = order[j - 1];
      order[j - 1] = t;
    }
  }
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), 0, 0, 0};
  cuuint64_t strides[3];
  cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / elem_bytes), 1u, 1u, 1u};
  int p = 0;
  for (int i = 0; i < 3; ++i) {
    dims[i + 1] = static_cast<cuuint64_t>(size[order[i]]);
    strides[i] = static_cast<cuuint64_t>(stride[order[i]]) * elem_bytes;
    if (order[i] == 0) box[i + 1] = static_cast<cuuint32_t>(rows);
    p |= i << (2 * order[i]);
  }
  const cuuint32_t estride[4] = {1u, 1u, 1u, 1u};
  const CUresult r = enc(m, dt, 4, const_cast<void*>(base), dims, strides, box, estride,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  *pos = p;
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

std::atomic<unsigned int> g_epoch_host{0};

int sm_count_of(int dev) {
  static std::atomic<int> cache[64];
  const int d = dev & 63;
  int n = cache[d].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      n = 148;
    }
    cache[d].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Tensor maps, kernel arguments and the persistent grid, shared by both kernels.
struct Prepared {
  alignas(64) CUtensorMap mq;
  alignas(64) CUtensorMap mk;
  alignas(64) CUtensorMap mv;
  alignas(64) CUtensorMap mo;  // O, 128-row boxes (kernels that store O by TMA)
  KArgs ka;
  int grid;
  int dev;
};

template <typename T>
cudaError_t prepare(const LaunchArgs& a, int D, int BN, Prepared* pr) {
  constexpr int kEB = static_cast<int>(sizeof(T));
  cudaError_t e = cudaGetDevice(&pr->dev);
  if (e != cudaSuccess) return e;
  const CUtensorMapDataType dt = std::is_same<T, __nv_bfloat16>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : std::is_same<T, float>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const long long hq = static_cast<long long>(a.B) * a.H;
  KArgs& ka = pr->ka;
  ka.o_pos = 0;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  if ((e = make_tmap(&pr->mq, a.q, dt, kEB, D, a.N, a.H, a.B, kBlockM, a.sq, sw, &ka.q_pos)) !=
      cudaSuccess) {
    return e;
  }
  if ((e = make_tmap(&pr->mk, a.k, dt, kEB, D, a.N, a.Hkv, a.B, BN, a.sk, sw, &ka.k_pos)) !=
      cudaSuccess) {
    return e;
  }
  // tf32 V is an MN-major operand: 32-byte swizzle atoms (see sdesc_sw128_atom32).
  const CUtensorMapSwizzle v_swizzle = kEB == 4 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : sw;
  if ((e = make_tmap(&pr->mv, a.v, dt, kEB, D, a.N, a.Hkv, a.B, BN, a.sv, v_swizzle, &ka.v_pos)) !=
      cudaSuccess) {
    return e;
  }
  if (kEB == 2 && (e = make_tmap(&pr->mo, a.o, dt, kEB, D, a.N, a.H, a.B, kBlockM, a.so, sw,
                                 &ka.o_pos)) != cudaSuccess) {
    return e;
  }
  ka.o = a.o;
  ka.o_sb = a.so[0];
  ka.o_sh = a.so[1];
  ka.o_sn = a.so[2];
  ka.lse = a.lse;
  ka.H = a.H;
  ka.Hkv = a.Hkv;
  ka.N = a.N;
  ka.n_q_tiles = (a.N + kBlockM - 1) / kBlockM;
  const long long items = hq * ka.n_q_tiles;
  if (hq > INT_MAX || items <= 0 || items > INT_MAX) return cudaErrorInvalidValue;
  ka.n_bh = static_cast<int>(hq);
  ka.n_items = static_cast<int>(items);
  // Heads per scheduling group: as many as keep their K+V within 48 MB of L2 (all of them when
  // everything fits).  With GQA a group's query heads share kv heads; counting K+V per query head
  // overestimates the footprint, which only makes groups smaller.
  const double kv_per_head = 2.0 * static_cast<double>(a.N) * D * kEB;
  const double kv_budget = 48.0 * 1024 * 1024;
  const long long fit = static_cast<long long>(kv_budget / kv_per_head);
  ka.head_group = static_cast<int>(fit >= hq ? hq : (fit < 1 ? 1 : fit));
  ka.scale = a.scale;
  ka.scale_log2 = a.scale * 1.4426950408889634f;
  ka.timeout_ns = a.timeout_ns;
  unsigned int ep = g_epoch_host.fetch_add(1) + 1;
  if (ep == 0) ep = g_epoch_host.fetch_add(1) + 1;
  ka.epoch = ep;
  ka.skip_kv_tile = a.skip_kv_tile;
  // Persistent grid: one CTA per SM (the kernels need a whole SM's TMEM and shared memory).
  const int sms = sm_count_of(pr->dev);
  pr->grid = static_cast<int>(items < sms ? items : sms);
  return cudaSuccess;
}

// Opts the kernel into its dynamic shared memory.  Done on every launch: the attribute belongs to
// the kernel as loaded in the current context, not to the device, so a flag remembered per device
// would be stale after cudaDeviceReset or for a caller running in a context of its own (a
// driver-API plugin); the call is a host-side attribute update and allocates nothing.
template <typename Kern>
cudaError_t opt_in_smem(Kern* kern, int bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <typename T, int D, int BN, int KST, int VST, bool CAUSAL>
cudaError_t launch_impl(const LaunchArgs& a, cudaStream_t stream) {
  using L = Layout<static_cast<int>(sizeof(T)), D, BN, KST, VST>;
  auto* kern = &fa_fwd_sm100_kernel<T, D, BN, KST, VST, CAUSAL>;
  Prepared pr;
  cudaError_t e = prepare<T>(a, D, BN, &pr);
  if (e != cudaSuccess) return e;
  if ((e = opt_in_smem(kern, L::kSmemAlloc)) != cudaSuccess) return e;
  kern<<<pr.grid, kThreads, L::kSmemAlloc, stream>>>(pr.mq, pr.mk, pr.mv, pr.mo, pr.ka);
  return cudaGetLastError();
}

// The 64-key lookahead kernel (fa_fwd_lookahead.cuh), fp16/bf16.
template <typename T, int D, bool CAUSAL>
cudaError_t launch_lookahead(const LaunchArgs& a, cudaStream_t stream) {
  // K and V rings of 128-key slots (32 KB at D=128, 16 KB at D=64) next to the Q tile.
  constexpr int kKSt = D == 128 ? 3 : 5;
  constexpr int kVSt = D == 128 ? 2 : 5;
  using L = LaLayout<D, kKSt, kVSt>;
  auto* kern = &fa_fwd_lookahead_kernel<T, D, kKSt, kVSt, CAUSAL, true>;
  Prepared pr;
  cudaError_t e = prepare<T>(a, D, L::BR, &pr);
  if (e != cudaSuccess) return e;
  if ((e = opt_in_smem(kern, L::kSmemAlloc)) != cudaSuccess) return e;
  kern<<<pr.grid, kThreads, L::kSmemAlloc, stream>>>(pr.mq, pr.mk, pr.mv, pr.mo, pr.ka);
  return cudaGetLastError();
}

// Ring depth for one key-tile width: as many K and V slots (up to 4 each) as fit next to the Q
// tile in ~200 KB of shared memory with one CTA per SM.
constexpr int ring_depth(int eb, int d, int bn) {
  return ((200 * 1024 - 128 * d * eb) / (2 * bn * d * eb)) < 4
             ? ((200 * 1024 - 128 * d * eb) / (2 * bn * d * eb))
             : 4;
}

template <typename T, int D, int BN, int KST, int VST>
cudaError_t launch_c(const LaunchArgs& a, cudaStream_t s) {
  return a.causal ? launch_impl<T, D, BN, KST, VST, true>(a, s)
                  : launch_impl<T, D, BN, KST, VST, false>(a, s);
}

template <typename T, int D>
cudaError_t launch_d(const LaunchArgs& a, cudaStream_t s) {
  constexpr int kEB = static_cast<int>(sizeof(T));
  if constexpr (kEB == 4) {
    // fp32 on tf32: 32- and 64-key tiles (and 128 at D=64), symmetric rings.
    switch (a.block_n) {
      case 64:
        return launch_c<T, D, 64, ring_depth(4, D, 64), ring_depth(4, D, 64)>(a, s);
      case 32:
        return launch_c<T, D, 32, ring_depth(4, D, 32), ring_depth(4, D, 32)>(a, s);
      case 128:
        if constexpr (D == 64) return launch_c<T, D, 128, 2, 2>(a, s);
        return cudaErrorInvalidValue;
      default:
        return cudaErrorInvalidValue;
    }
  } else {
    // D=128, BN=128: 3 K slots + 2 V slots of 32 KB next to the 32 KB Q tile.
    constexpr int kKSt128 = (D == 128) ? 3 : 4;
    constexpr int kVSt128 = (D == 128) ? 2 : 4;
    switch (a.block_n) {
      case 128:
        return launch_c<T, D, 128, kKSt128, kVSt128>(a, s);
      case 64:
        return a.causal ? launch_lookahead<T, D, true>(a, s) : launch_lookahead<T, D, false>(a, s);
      case 32:
        return launch_c<T, D, 32, 4, 4>(a, s);
      default:
        return cudaErrorInvalidValue;
    }
  }
}

// fp32: round q/k/v into the workspace, then run the tf32 kernel on the rounded copies.
cudaError_t launch_f32(const LaunchArgs& a, cudaStream_t s);

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
  if (dtype == FA_DTYPE_F32) return block_n == 32 || block_n == 64 || (block_n == 128 && D == 64);
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return false;
  return block_n == 32 || block_n == 64 || block_n == 128;
}

// Default key-tile choice: the lookahead kernel (128-key rounds split 64/64 between the softmax
// warpgroups, selected by block_n = 64) for D = 128 and for causal attention at D = 64; the
// 128-key kernel for full attention at D = 64, where the lookahead kernel's per-round overheads
// weigh more against the shorter MMAs.  Measured on B200 (TFLOP/s, 128-key / lookahead): fp16
// causal D=64 B8H32 N512-4096 175/199 .. 550/562, the GPT-2 block's B16H12 N1024 300/331, C2c
// 280/299, N=8192 604/599; bf16 causal D=64 B8H32 N2048 381/408, B16H12 N1024 260/292, C2c
// 261/262; fp16 full D=64 C2 400/399, B8H32 N2048 607/607; bf16 full D=64 C2 399/380, B8H32
// N2048 575/548.  fp32 runs 64-key tf32 tiles.
int default_block_n(int dtype, int D, int /*N*/, int causal) {
  if (dtype == FA_DTYPE_F32) return 64;
  if (D == 128) return 64;
  return causal ? 64 : 128;
}

cudaError_t launch_forward(const LaunchArgs& a, cudaStream_t stream) {
  switch (a.dtype) {
    case FA_DTYPE_F16:
      return launch_t<__half>(a, stream);
    case FA_DTYPE_BF16:
      return launch_t<__nv_bfloat16>(a, stream);
    case FA_DTYPE_F32:
      return launch_f32(a, stream);
    default:
      return cudaErrorNotSupported;
  }
}

namespace {
cudaError_t launch_f32(const LaunchArgs& a, cudaStream_t s) {
  if (a.workspace == nullptr) return cudaErrorInvalidValue;
  const int d4 = a.D / 4;  // 16-byte units per row
  const size_t nq = static_cast<size_t>(a.B) * a.H * a.N * d4;
  const size_t nkv = static_cast<size_t>(a.B) * a.Hkv * a.N * d4;
  uint4* ws = static_cast<uint4*>(a.workspace);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const View4 vq{static_cast<const float*>(a.q), a.sq[0], a.sq[1], a.sq[2], a.H, nq};
  const View4 vk{static_cast<const float*>(a.k), a.sk[0], a.sk[1], a.sk[2], a.Hkv, nkv};
  const View4 vv{static_cast<const float*>(a.v), a.sv[0], a.sv[1], a.sv[2], a.Hkv, nkv};
  const size_t n = nq + 2 * nkv;
  const size_t want = (n + 255) / 256;
  const size_t cap = static_cast<size_t>(sm_count_of(dev)) * 8;
  const unsigned int grid = static_cast<unsigned int>(want < cap ? want : cap);
  fa_round_tf32_kernel<<<grid, 256, 0, s>>>(vq, vk, vv, a.N, d4, ws);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  // The kernel then reads the contiguous copies; o keeps the caller's strides.
  LaunchArgs r = a;
  r.q = ws;
  r.k = ws + nq;
  r.v = ws + nq + nkv;
  const long long nd = static_cast<long long>(a.N) * a.D;
  const long long cq[3] = {static_cast<long long>(a.H) * nd, nd, a.D};
  const long long ckv[3] = {static_cast<long long>(a.Hkv) * nd, nd, a.D};
  for (int i = 0; i < 3; ++i) {
    r.sq[i] = cq[i];
    r.sk[i] = ckv[i];
    r.sv[i] = ckv[i];
  }
  return launch_t<float>(r, s);
}
}  // namespace

size_t workspace_bytes_f32(int B, int H, int Hkv, int N, int D) {
  return 4ull * static_cast<size_t>(D) * static_cast<size_t>(N) *
         (static_cast<size_t>(B) * H + 2ull * static_cast<size_t>(B) * Hkv);
}

#ifdef FA_TRACE
extern "C" int fa_debug_read_trace(long long* out, long long* t0) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(out, g_trace, sizeof(g_trace));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(t0, g_trace_t0, sizeof(g_trace_t0));
  return static_cast<int>(e);
}
#endif

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
  if (v == 0) return cudaSuccess;
  return (v & kStBounds) != 0 ? cudaErrorAssert : cudaErrorLaunchTimeout;
}

}  // namespace fa_sm100
