// fa_fwd_lookahead.cuh -- sm_100a SDPA forward for fp16/bf16: 128-key rounds split by columns
// between the two softmax warpgroups, P in its own tensor-memory columns, Q held in tensor memory,
// and the next round's S computed while the softmax works on the current one.  Included by
// fa_fwd_sm100.cu after fa_kernel_common.cuh (one translation unit).
//
// Same work decomposition, warp roles, numerics and failure handling as the kernel in
// fa_fwd_sm100.cu: persistent CTAs over (head, 128-row query tile) items; warp 0 loads Q and K,
// warp 2 loads V, lane 0 of warp 1 issues the S MMAs and lane 0 of warp 3 the PV MMAs (two issuing
// threads: a thread's mbarrier waits do not overlap its own queued MMAs); two softmax warpgroups run
// the online softmax on disjoint key sets and their partial results are merged at the end like
// split-KV partials.  The layout differs:
//
//   tensor memory columns (lane = query row):
//     Q     [0, D/2)                    16-bit, two per column: the A operand of S = Q K^T
//     S     D/2 .. D/2+128              fp32 scores of the round's 128 keys;
//                                       warpgroup g reads keys 64g .. 64g+63 (columns D/2 + 64g)
//     P_g   D/2 + 128 + 32g .. +32      16-bit weights of warpgroup g: A operand of O_g += P_g V_g
//     O_g   D/2 + 192 + gD .. +D        fp32 accumulators
//   (D = 128: exactly the 512 columns of an SM.)
//
// One round = one 128-key tile of K and V (one ring slot each).  Per round the tensor core runs
// S(r) = Q K_r^T (8 M=128 N=128 K=16 MMAs, Q from tensor memory) and PV_0(r), PV_1(r) (4 MMAs each,
// V rows 0-63 and 64-127 of the slot): 16 MMAs at the full N=128 rate, 4 commits, 4 barrier waits.
// Because P_g has its own columns, S(r+1) may overwrite S as soon as both warpgroups have LOADED
// S(r) into registers (barrier s_free); the softmax waits for PV(r-1) (barrier pv_done) only right
// before it stores P_g(r).  S(x) is issued once both warpgroups have loaded S(x-1) (and, after a bf16
// first-causal-tile item, where P is carried as P_hi + P_lo with P_lo stored over S, once that
// round's PVs have completed); PV_g(r) once P_g(r) is stored.  So while the warpgroups compute
// P(r+1) from S(r+1), the tensor core runs PV(r) and S(r+2).
// Q(i+1) replaces Q(i) in tensor memory once the S MMAs of item i have completed (q_done); the
// copy is tcgen05.cp from the TMA-loaded shared-memory tile.
//
// A round past the valid keys of an item (N not a multiple of 128, or the causal diagonal) is
// still a full 128-key round: TMA zero-fills rows past N and the softmax masks every score past
// the row's last visible key to -inf, so those weights are exactly 0.
#pragma once

#include "fa_kernel_common.cuh"

namespace fa_sm100 {
namespace {

template <int D, int KST, int VST>
struct LaLayout {
  static constexpr int BR = 128;                 // keys per round (one K/V ring slot)
  static constexpr int BG = 64;                  // keys per warpgroup per round
  static constexpr int kQChunkBytes = kBlockM * 128;
  static constexpr int kKVChunkBytes = BR * 128;
  static constexpr int kQBytes = kBlockM * D * 2;
  static constexpr int kKVBytes = BR * D * 2;
  static constexpr int kDChunks = D / 64;        // 128-byte column chunks along D
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + KST * kKVBytes;
  // O staging for the TMA store of the epilogue: kDChunks 128-byte-swizzled 128-row chunks, like
  // the Q tile.  The merge's (m, l) exchange lives at its start: it is read before O is staged.
  static constexpr int kOStOff = kVOff + VST * kKVBytes;
  static constexpr int kOStBytes = kBlockM * D * 2;
  static constexpr int kXchOff = kOStOff;
  static constexpr int kXchBytes = 2 * 2 * kBlockM * 4 + 16;
  static constexpr int kBarOff = kOStOff + kOStBytes;

  // Barrier indices.
  static constexpr int kBarQFull = 0;   // TMA: Q tile landed in shared memory
  static constexpr int kBarQFree = 1;   // Q's shared-memory buffer may be reloaded
  static constexpr int kBarQDone = 2;   // the item's S MMAs completed (Q in TMEM may change)
  static constexpr int kBarSFull = 3;   // S(r) computed
  static constexpr int kBarSFree = 4;   // S(r) loaded by both warpgroups (256 arrivals)
  static constexpr int kBarPFull = 5;   // + g: P_g(r) stored (128 arrivals)
  static constexpr int kBarPVDone = 7;  // + g: PV_g(r) completed (P_g free, O_g updated)
  static constexpr int kBarExp = 9;     // + g: warpgroup g finished its exponentials (128)
  static constexpr int kBarOFree = 11;  // epilogue has read O_0 and O_1 (256 arrivals)
  static constexpr int kBarDrain = 12;  // + issuer (S side 0, PV side 1)
  static constexpr int kBarKFull = 14;
  static constexpr int kBarKEmpty = kBarKFull + KST;
  static constexpr int kBarVFull = kBarKEmpty + KST;
  static constexpr int kBarVEmpty = kBarVFull + VST;
  static constexpr int kNumBars = kBarVEmpty + VST;
  static constexpr int kMiscOff = kBarOff + 8 * kNumBars;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kSmemAlloc = kBytes + 1024;

  // Tensor memory columns.
  static constexpr int kColQ = 0;
  static constexpr int kColS = D / 2;            // + g * BG for warpgroup g's keys
  static constexpr int kColP = D / 2 + BR;       // + g * BG / 2
  static constexpr int kColO = D / 2 + BR + BG;  // + g * D
  static constexpr int kColsUsed = kColO + 2 * D;
  static constexpr int kTmemCols = kColsUsed <= 256 ? 256 : 512;

  static_assert(D == 64 || D == 128, "head dim");
  static_assert(kColsUsed <= 512, "tensor memory overflow");
  static_assert(kSmemAlloc <= 232448, "shared memory overflow");
  static_assert(kXchBytes <= kOStBytes, "exchange must fit inside the O staging buffer");
};

// Walks the CTA's items round by round.
template <bool CAUSAL>
struct RoundCursor {
  int local;  // CTA-local item ordinal
  int item;   // global item index, -1 past the end
  int n_rounds, rr;
  bool comp;  // bf16 first causal query tile: P carried as P_hi + P_lo

  __device__ __forceinline__ void seek(int l, int G, int cta, const KArgs& a, bool bf16) {
    local = l;
    rr = 0;
    const int i = item_index(l, G, cta);
    if (i >= a.n_items) {
      item = -1;
      n_rounds = 0;
      comp = false;
      return;
    }
    item = i;
    const Item it = decode_item<CAUSAL>(i, a);
    const int q0 = it.q_tile * kBlockM;
    const int kv_end = CAUSAL ? min(a.N, q0 + kBlockM) : a.N;
    n_rounds = (kv_end + 127) / 128;
    comp = bf16 && CAUSAL && it.q_tile == 0;
  }
  __device__ __forceinline__ void next(int G, int cta, const KArgs& a, bool bf16) {
    if (++rr == n_rounds) seek(local + 1, G, cta, a, bf16);
  }
};

// Whether the two softmax warpgroups take turns on the exponentials (build-time switch, off by
// default: with one S buffer the lagging warpgroup delays s_free, and with it the next S, by more
// than the overlap gains -- measured 922 vs 986 TFLOP/s at N=8192).
#ifndef FA_EXP_TURNS
#define FA_EXP_TURNS 0
#endif
constexpr bool kExpTurns = FA_EXP_TURNS != 0;

// Opaque to the compiler: code that uses `x` afterwards cannot be moved above this point.
__device__ __forceinline__ void launder(float& x) { asm volatile("" : "+f"(x)); }

// mbarrier arrive that the compiler may only issue once `dep` has been computed.
__device__ __forceinline__ void mbar_arrive_after(uint32_t bar, float dep) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar), "f"(dep) : "memory");
}

// Every kLaEmuEvery-th pair of exponentials is computed on the FMA pipes (ex2_poly3) instead of
// the MUFU unit, which both warpgroups saturate during their exponential phase (15.6 exp2/clk/SM
// measured).  One pair in four measured best on B200 (C3 557 vs 524 TFLOP/s, N=8192 1037 vs 980;
// one in three or two is slower).  Build-time switch FA_LA_EX2_EMU_EVERY (0 = all on MUFU).
#ifndef FA_LA_EX2_EMU_EVERY
#define FA_LA_EX2_EMU_EVERY 4
#endif
constexpr int kLaEmuEvery = FA_LA_EX2_EMU_EVERY;

// p = 2^(s*c - m*c) for the 64 columns of one S row, packed two per 32-bit word into pk[32]
// (and P_lo = p - round(p) into lo[32] when kLo); returns the sum of the fp32 weights.
template <typename T, bool kLo>
__device__ __forceinline__ float exp_pack64(const float (&s)[64], float sl2, float mc,
                                            uint32_t (&pk)[32], uint32_t (&lo)[32]) {
  const uint64_t c2 = f2_pack(sl2, sl2);
  const uint64_t nb2 = f2_pack(-mc, -mc);
  uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const uint64_t x = f2_fma(f2_pack(s[2 * c], s[2 * c + 1]), c2, nb2);
    float p0, p1;
    constexpr int kE = kLaEmuEvery > 0 ? kLaEmuEvery : 1;
    if (kLaEmuEvery > 0 && (c % kE) == kE - 1) {
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
  const uint64_t t = f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
  return f2_lo(t) + f2_hi(t);
}

// bf16 with P carried as P_hi + P_lo: the exponentials of the 64 columns, P_hi stored at `p_addr`
// and P_lo at `lo_addr`, eight columns at a time.  Only the first causal query tile runs it, so it
// is a separate (not inlined) function reading the row from a stack copy: inlined, its extra live
// words raise the register allocation of the whole kernel from 127 to 159-167 and slow every
// round of bf16 causal launches by 6-9% (measured).  Returns the sum of the fp32 weights.
template <typename T>
__device__ __noinline__ float exp_pack64_hilo_store(const float* s, float sl2, float mc,
                                                    uint32_t p_addr, uint32_t lo_addr) {
  const uint64_t c2 = f2_pack(sl2, sl2);
  const uint64_t nb2 = f2_pack(-mc, -mc);
  uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll 1
  for (int c0 = 0; c0 < 32; c0 += 8) {
    uint32_t pk[8], lo[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int cc = c0 + c;
      const uint64_t x = f2_fma(f2_pack(s[2 * cc], s[2 * cc + 1]), c2, nb2);
      const float p0 = ex2_approx(f2_lo(x));
      const float p1 = ex2_approx(f2_hi(x));
      pk[c] = pack2<T>(p0, p1);
      acc[c & 3] = f2_add(acc[c & 3], f2_pack(p0, p1));
      lo[c] = pack2<T>(p0 - __uint_as_float(pk[c] << 16), p1 - __uint_as_float(pk[c] & 0xFFFF0000u));
    }
    tmem_st8(p_addr + c0, pk);
    tmem_st8(lo_addr + c0, lo);
  }
  const uint64_t t = f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
  return f2_lo(t) + f2_hi(t);
}

// PV of a bf16 first-causal-tile round (the item's only round, accumulate = 0): for each warpgroup
// g, once its P is stored, O_g = P_hi,g V_g + P_lo,g V_g.  Not inlined (see the PV issuer).
template <typename L, uint32_t kIdescPV>
__device__ __noinline__ bool issue_pv_hilo(uint32_t tmem, uint64_t v_desc, uint32_t bar_pfull,
                                           uint32_t bar_pvdone, uint32_t parity, const WaitCtx& w) {
  constexpr int BG = L::BG;
  for (int g = 0; g < 2; ++g) {
    if (!wait_bounded(bar_pfull + 8u * g, parity, w, kStPFull)) return false;
    tc_fence_after();
    const uint64_t vg = v_desc + static_cast<uint64_t>((g * BG * 128) >> 4);
    const uint32_t o_tmem = tmem + L::kColO + g * L::kDChunks * 64;
    const uint32_t pa = tmem + L::kColP + g * (BG / 2);
    const uint32_t plo = tmem + L::kColS + g * BG;
#pragma unroll
    for (int kk = 0; kk < BG / 16; ++kk) {
      umma_ts(o_tmem, pa + kk * 8, vg + ((kk * 16 * 128) >> 4), kIdescPV, kk > 0 ? 1u : 0u);
    }
#pragma unroll
    for (int kk = 0; kk < BG / 16; ++kk) {
      umma_ts(o_tmem, plo + kk * 8, vg + ((kk * 16 * 128) >> 4), kIdescPV, 1u);
    }
    umma_commit(bar_pvdone + 8u * g);
  }
  return true;
}

template <typename T, int D, int KST, int VST, bool CAUSAL, bool QTMEM>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_lookahead_kernel(const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v,
                            const __grid_constant__ CUtensorMap tm_o, const KArgs args) {
  using L = LaLayout<D, KST, VST>;
  constexpr int BR = L::BR;
  constexpr int BG = L::BG;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kFmt = kBf16 ? 1u : 0u;
  // Rescale threshold (log2 units).  fp16 P keeps 11 significant bits, so weights up to 2^8
  // (lazy rescaling) cost nothing; bf16 keeps 8, and a row's largest weight must stay exactly 1
  // (rescale whenever the running max grows) or its rounding error reaches the 8e-3 gate.
  constexpr float kResc = kBf16 ? 0.0f : kRescaleThreshold;

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
    mbar_init(bar(L::kBarQFree), 1);
    mbar_init(bar(L::kBarQDone), 1);
    mbar_init(bar(L::kBarSFull), 1);
    mbar_init(bar(L::kBarSFree), 2 * kBlockM);
    for (int g = 0; g < 2; ++g) {
      mbar_init(bar(L::kBarPFull + g), kBlockM);
      mbar_init(bar(L::kBarPVDone + g), 1);
      mbar_init(bar(L::kBarExp + g), kBlockM);
    }
    mbar_init(bar(L::kBarOFree), 2 * kBlockM);
    mbar_init(bar(L::kBarDrain), 1);
    mbar_init(bar(L::kBarDrain + 1), 1);
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
      tma_load_view(sbase + L::kQOff + c * L::kQChunkBytes, &tm_q, c * 64, it0.q_tile * kBlockM,
                    hd0.h, hd0.b, args.q_pos, bar(L::kBarQFull));
    }
    pre_k = min(KST, (kv_end0 + BR - 1) / BR);
    for (int j = 0; j < pre_k; ++j) {
      if (j == args.skip_kv_tile) continue;
      mbar_arrive_expect_tx(bar(L::kBarKFull + j), L::kKVBytes);
#pragma unroll
      for (int c = 0; c < L::kDChunks; ++c) {
        tma_load_view(sbase + L::kKOff + j * L::kKVBytes + c * L::kKVChunkBytes, &tm_k, c * 64,
                      j * BR, hd0.hk, hd0.b, args.k_pos, bar(L::kBarKFull + j));
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
    // warp 0: Q of every item and the K ring; warp 2: the V ring (one 128-key tile per slot).
    if (lane == 0) {
      const bool is_k = (warp == 0);
      const int nst = is_k ? KST : VST;
      const int bar_full = is_k ? L::kBarKFull : L::kBarVFull;
      const int bar_empty = is_k ? L::kBarKEmpty : L::kBarVEmpty;
      const uint32_t ring = sbase + (is_k ? L::kKOff : L::kVOff);
      const CUtensorMap* tm = is_k ? &tm_k : &tm_v;
      if (!is_k) tma_prefetch_desc(tm);
      int count = 0;
      int items_done = 0;
      unsigned skipped = 0;
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int i = item_index(r, G, cta);
        if (i >= args.n_items) break;
        const Item item = decode_item<CAUSAL>(i, args);
        const int q0 = item.q_tile * kBlockM;
        const Heads hd = split_heads(item.bh, args);
        const int kv_end = CAUSAL ? min(args.N, q0 + kBlockM) : args.N;
        const int n_rounds = (kv_end + BR - 1) / BR;
        if (is_k) {
          // The previous item's Q must have left the shared-memory buffer.
          if (items_done > 0 &&
              !(ok = wait_bounded(bar(L::kBarQFree), static_cast<uint32_t>(items_done - 1) & 1u,
                                  w, kStKVEmpty))) {
            break;
          }
          if (items_done > 0) {  // the first item's Q went out in the prologue
            mbar_arrive_expect_tx(bar(L::kBarQFull), L::kQBytes);
#pragma unroll
            for (int c = 0; c < L::kDChunks; ++c) {
              tma_load_view(sbase + L::kQOff + c * L::kQChunkBytes, &tm_q, c * 64, q0, hd.h, hd.b,
                            args.q_pos, bar(L::kBarQFull));
            }
          }
          ++items_done;
        }
        for (int j = 0; j < n_rounds; ++j, ++count) {
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
            tma_load_view(ring + s * L::kKVBytes + c * L::kKVChunkBytes, tm, c * 64, j * BR, hd.hk,
                          hd.b, is_k ? args.k_pos : args.v_pos, bar(bar_full + s));
          }
        }
      }
      if (is_k && items_done > 0) {
        wait_drain(bar(L::kBarQFull), static_cast<uint32_t>(items_done - 1) & 1u, args.timeout_ns);
      }
      for (int c = (count > nst ? count - nst : 0); c < count; ++c) {
        if (!((skipped >> (c & 31)) & 1u)) {
          wait_drain(bar(bar_full + c % nst), static_cast<uint32_t>(c / nst) & 1u, args.timeout_ns);
        }
      }
    }
  } else if (warp == 1 || warp == 3) {
    // ------------------------------------------------------------------ MMA issuers
    // Lane 0 of warp 1 issues Q's copy into tensor memory and the S MMAs; lane 0 of warp 3 the PV
    // MMAs.  tcgen05.commit tracks the issuing thread's own operations, so each keeps its own
    // barriers; the only ordering between the two streams is through barriers.
    if (lane == 0) {
      const bool s_side = (warp == 1);
      RoundCursor<CAUSAL> cur;
      cur.seek(0, G, cta, args, kBf16);
      bool ok = true;
      if (s_side) {
        constexpr uint32_t kIdescS = idesc_mma(kFmt, kBlockM, BR, false);
        const uint64_t q_desc0 = sdesc_sw128(sbase + L::kQOff, 16, 1024);
        const uint64_t k_desc0 = sdesc_sw128(sbase + L::kKOff, 16, 1024);
        int s_cnt = 0;      // S rounds issued, over all items
        int q_staged = 0;   // items whose Q was staged
        bool prev_comp = false;
        while (ok && cur.item >= 0) {
          if (cur.rr == 0) {
            // First S of an item: stage its Q.
            if constexpr (QTMEM) {
              if (q_staged > 0 &&
                  !(ok = wait_bounded(bar(L::kBarQDone), static_cast<uint32_t>(q_staged - 1) & 1u,
                                      w, kStQFull))) {
                break;
              }
            }
            if (!(ok = wait_bounded(bar(L::kBarQFull), static_cast<uint32_t>(q_staged) & 1u, w,
                                    kStQFull))) {
              break;
            }
            tc_fence_after();
            if constexpr (QTMEM) {
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t q_off = (kk / 4) * L::kQChunkBytes + (kk % 4) * 32;
                tmem_cp_128x256b(tmem + L::kColQ + kk * 8, q_desc0 + (q_off >> 4));
              }
              umma_commit(bar(L::kBarQFree));
              // The copy must have landed before an MMA reads Q from tensor memory.
              if (!(ok = wait_bounded(bar(L::kBarQFree), static_cast<uint32_t>(q_staged) & 1u, w,
                                      kStQFull))) {
                break;
              }
              tc_fence_after();
            }
            ++q_staged;
          }
          FA_TRACE_EV(cur.local == 0, 4, 0, cur.rr);
          if (s_cnt > 0) {
            // Both warpgroups have S(x-1) in registers.
            const uint32_t par = static_cast<uint32_t>(s_cnt - 1) & 1u;
            if (!(ok = wait_bounded(bar(L::kBarSFree), par, w, kStSFree))) break;
            FA_TRACE_EV(cur.local == 0, 5, 0, cur.rr);
            if (prev_comp) {
              // P_lo of the previous round lives in S until both PVs have read it.
              if (!(ok = wait_bounded(bar(L::kBarPVDone + 0), par, w, kStSFree))) break;
              if (!(ok = wait_bounded(bar(L::kBarPVDone + 1), par, w, kStSFree))) break;
            }
          }
          const int s = s_cnt % KST;
          if (!(ok = wait_bounded(bar(L::kBarKFull + s), static_cast<uint32_t>(s_cnt / KST) & 1u, w,
                                  kStKFull))) {
            break;
          }
          tc_fence_after();
          FA_TRACE_EV(cur.local == 0, 0, 0, cur.rr);
          const uint32_t d_tmem = tmem + L::kColS;
          const uint64_t k_desc = k_desc0 + static_cast<uint64_t>((s * L::kKVBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t k_off = (kk / 4) * L::kKVChunkBytes + (kk % 4) * 32;
            if constexpr (QTMEM) {
              umma_ts(d_tmem, tmem + L::kColQ + kk * 8, k_desc + (k_off >> 4), kIdescS,
                      kk > 0 ? 1u : 0u);
            } else {
              const uint32_t q_off = (kk / 4) * L::kQChunkBytes + (kk % 4) * 32;
              umma_ss(d_tmem, q_desc0 + (q_off >> 4), k_desc + (k_off >> 4), kIdescS,
                      kk > 0 ? 1u : 0u);
            }
          }
          FA_TRACE_EV(cur.local == 0, 4, 1, cur.rr);
          umma_commit(bar(L::kBarSFull));
          umma_commit(bar(L::kBarKEmpty + s));
          if (cur.rr == cur.n_rounds - 1) {
            // The item's last S: Q (TMEM copy, or the shared-memory tile) is no longer read.
            umma_commit(bar(QTMEM ? L::kBarQDone : L::kBarQFree));
          }
          prev_comp = cur.comp;
          ++s_cnt;
          cur.next(G, cta, args, kBf16);
        }
      } else {
        constexpr uint32_t kIdescPV = idesc_mma(kFmt, kBlockM, D, true);
        const uint64_t v_desc0 = sdesc_sw128(sbase + L::kVOff, L::kKVChunkBytes, 1024);
        int pv_cnt = 0;  // PV rounds issued, over all items
        while (ok && cur.item >= 0) {
          if (cur.rr == 0 && cur.local > 0 &&
              !(ok = wait_bounded(bar(L::kBarOFree), static_cast<uint32_t>(cur.local - 1) & 1u, w,
                                  kStODone))) {
            break;
          }
          const int s = pv_cnt % VST;
          if (!(ok = wait_bounded(bar(L::kBarVFull + s), static_cast<uint32_t>(pv_cnt / VST) & 1u,
                                  w, kStVFull))) {
            break;
          }
          const uint64_t v_desc = v_desc0 + static_cast<uint64_t>((s * L::kKVBytes) >> 4);
          if (kBf16 && cur.comp) {
            // The first causal query tile (bf16), a single round: P_hi then P_lo (over the
            // warpgroup's S columns).  Kept apart from the common round below, whose issue code
            // measured ~8% faster without the P_lo block inside it (C4, bf16).
            ok = issue_pv_hilo<L, kIdescPV>(tmem, v_desc, bar(L::kBarPFull), bar(L::kBarPVDone),
                               static_cast<uint32_t>(pv_cnt) & 1u, w);
          } else {
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              // Each warpgroup's PV goes as soon as its own P is stored.
              if (!(ok = wait_bounded(bar(L::kBarPFull + g), static_cast<uint32_t>(pv_cnt) & 1u, w,
                                      kStPFull))) {
                break;
              }
              tc_fence_after();
              FA_TRACE_EV(cur.local == 0, 1, g, cur.rr);
              // Warpgroup g's keys are rows 64g .. 64g+63 of the V slot.
              const uint64_t vg = v_desc + static_cast<uint64_t>((g * BG * 128) >> 4);
              const uint32_t o_tmem = tmem + L::kColO + g * D;
              const uint32_t pa = tmem + L::kColP + g * (BG / 2);
#pragma unroll
              for (int kk = 0; kk < BG / 16; ++kk) {
                umma_ts(o_tmem, pa + kk * 8, vg + ((kk * 16 * 128) >> 4), kIdescPV,
                        (cur.rr > 0 || kk > 0) ? 1u : 0u);
              }
              umma_commit(bar(L::kBarPVDone + g));
            }
          }
          if (!ok) break;
          umma_commit(bar(L::kBarVEmpty + s));
          ++pv_cnt;
          cur.next(G, cta, args, kBf16);
        }
      }
      // Exit path: every tcgen05 operation this thread issued must be complete before TMEM is
      // freed.
      const int drain = s_side ? L::kBarDrain : L::kBarDrain + 1;
      umma_commit(bar(drain));
      wait_drain(bar(drain), 0u, args.timeout_ns);
    }
    __syncwarp();
  } else if (warp >= kSoftmaxWarp0) {
    // ------------------------------------------------------------------ softmax warpgroups
    const int g = (warp - kSoftmaxWarp0) >> 2;  // keys 64g .. 64g+63 of every round
    const int r = (warp & 3) * 32 + lane;       // row within the tile == TMEM lane
    const uint32_t tl = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_col = L::kColS + g * BG;
    const uint32_t p_col = L::kColP + g * (BG / 2);
    const uint32_t o_col = L::kColO + g * D;
    const float sl2 = args.scale_log2;
    float* xch = reinterpret_cast<float*>(smem + L::kXchOff);
    volatile int* xch_ctl = reinterpret_cast<volatile int*>(smem + L::kXchOff + 2 * 2 * kBlockM * 4);
    const bool o_issuer = (g == 0 && warp == kSoftmaxWarp0 && lane == 0);  // O's TMA stores
    if (o_issuer) tma_prefetch_desc(&tm_o);
    int sc = 0;   // S rounds consumed, over all items
    int pvc = 0;  // PV rounds waited for, over all items
    int ec = 0;   // exponential phases run by this warpgroup, over all items
    for (int rnd = 0;; ++rnd) {
      const int i = item_index(rnd, G, cta);
      if (i >= args.n_items) break;
      const Item item = decode_item<CAUSAL>(i, args);
      (void)FA_DCHECK(item.bh < args.n_bh && item.q_tile >= 0 && item.q_tile < args.n_q_tiles);
      const int q0 = item.q_tile * kBlockM;
      const int row = q0 + r;
      const int kv_end = CAUSAL ? min(args.N, q0 + kBlockM) : args.N;
      const int n_rounds = (kv_end + BR - 1) / BR;
      const bool comp = kBf16 && CAUSAL && item.q_tile == 0;
      float m_ref = -INFINITY;
      float l_sum = 0.f;
      bool ok = true;
      for (int t = 0; t < n_rounds; ++t) {
        ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarSFull),
                                                  static_cast<uint32_t>(sc) & 1u, w, kStSFull));
        if (!ok) break;
        ++sc;
        tc_fence_after();
        FA_TRACE_EV(rnd == 0 && r == 0, 2, g, t);
        float s[BG];
        if (FA_DCHECK(s_col + BG <= L::kTmemCols)) load_s_row<BG>(tl + s_col, s);
        // S is in registers: the tensor core may compute the next round into it.
        tc_fence_before();
        mbar_arrive(bar(L::kBarSFree));
        const int kv0 = t * BR + g * BG;
        if ((CAUSAL && kv0 + BG - 1 > q0) || kv0 + BG > kv_end) {
          // Key kv0 + c is visible to this row iff c <= lim (top-left causal, inside kv_end): one
          // compare per score against a per-thread bound (measured +3-6 % on causal shapes with
          // many short items against the per-key index test it replaces).
          const int lim = (CAUSAL ? min(row, kv_end - 1) : kv_end - 1) - kv0;
#pragma unroll
          for (int c = 0; c < BG; ++c) s[c] = (c > lim) ? -INFINITY : s[c];
        }
        const float m_new = fmaxf(m_ref, row_max<BG>(s));
        const bool resc = (m_ref == -INFINITY) ? (m_new != -INFINITY)
                                               : ((m_new - m_ref) * sl2 > kResc);
        const float m_use = resc ? m_new : m_ref;
        const float alpha =
            resc ? ((m_ref == -INFINITY) ? 0.f : ex2_approx((m_ref - m_use) * sl2)) : 1.f;
        float mc = (m_use == -INFINITY) ? 0.f : m_use * sl2;
        // The two warpgroups take turns on the exponentials (the MUFU unit is shared): warpgroup 1
        // waits for warpgroup 0's phase of this round, warpgroup 0 for warpgroup 1's previous
        // one, so one group's loads, max and stores run under the other's exponentials.
        if (kExpTurns && (g == 1 || ec > 0)) {
          const uint32_t par = static_cast<uint32_t>(g == 1 ? ec : ec - 1) & 1u;
          ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarExp + (1 - g)), par, w, kStPFree));
          if (!ok) break;
        }
        ++ec;
        launder(mc);  // the exponentials may not start before the turn
        uint32_t pk[32], lo[32];
        float rs;
        if (kBf16 && comp) {
          // P_hi + P_lo (P_lo over the warpgroup's S columns, whose round is in registers).  The
          // first causal query tile has a single round (t == 0), so nothing reads P_g or S yet:
          // both go to tensor memory as they are computed.
          float s_copy[64];
#pragma unroll
          for (int c = 0; c < 64; ++c) s_copy[c] = s[c];
          rs = exp_pack64_hilo_store<T>(s_copy, sl2, mc, tl + p_col, tl + s_col);
        } else {
          rs = exp_pack64<T, false>(s, sl2, mc, pk, lo);
        }
        if (kExpTurns) mbar_arrive_after(bar(L::kBarExp + g), rs);  // turn passes on
        l_sum = l_sum * alpha + rs;
        m_ref = m_use;
        if (t > 0) {
          // PV_g(t-1) must be done with P_g (and with O_g, before a correction).
          ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarPVDone + g),
                                                    static_cast<uint32_t>(pvc) & 1u, w, kStPFree));
          if (!ok) break;
          ++pvc;
          tc_fence_after();
          if (__any_sync(0xffffffffu, resc) && FA_DCHECK(o_col + D <= L::kTmemCols)) {
            // 64 columns per wait: two loads in flight, then both scaled and stored back.
#pragma unroll
            for (int c = 0; c < D; c += 64) {
              uint32_t u[32], v[32];
              tmem_ld32_nowait(tl + o_col + c, u);
              tmem_ld32_nowait(tl + o_col + c + 32, v);
              tmem_wait_ld_regs(u);
              tmem_wait_ld_regs(v);
#pragma unroll
              for (int k2 = 0; k2 < 32; ++k2) {
                u[k2] = __float_as_uint(__uint_as_float(u[k2]) * alpha);
                v[k2] = __float_as_uint(__uint_as_float(v[k2]) * alpha);
              }
              tmem_st32(tl + o_col + c, u);
              tmem_st32(tl + o_col + c + 32, v);
            }
          }
        }
        if (!(kBf16 && comp) && FA_DCHECK(p_col + BG / 2 <= L::kTmemCols)) {
          tmem_st16(tl + p_col, &pk[0]);
          tmem_st16(tl + p_col + 16, &pk[16]);
        }
        tmem_st_wait();
        tc_fence_before();
        FA_TRACE_EV(rnd == 0 && r == 0, 3, g, t);
        mbar_arrive(bar(L::kBarPFull + g));
      }
      // ---- merge the two partials; O / l staged in shared memory and written by TMA; LSE ----
      // The previous item's O store must have read the staging buffer (the exchange lives there).
      if (o_issuer) bulk_wait_read();
      tc_fence_before();
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
      if (g == 0 && in_range && FA_DCHECK(item.bh < args.n_bh)) {
        args.lse[static_cast<size_t>(item.bh) * static_cast<size_t>(args.N) + static_cast<size_t>(row)] =
            (l > 0.f && m != -INFINITY) ? fmaf(m, args.scale, logf(l)) : INFINITY;
      }
      // The item's last PVs: waited for only now, so that the exchange above runs under them.  A
      // wait that runs out here does not leave the epilogue (every thread still reaches its
      // named barriers); the abort flag it sets ends the next item's first wait.
      if (ok) {
        ok = __all_sync(0xffffffffu, wait_bounded(bar(L::kBarPVDone + g),
                                                  static_cast<uint32_t>(pvc) & 1u, w, kStODone));
        ++pvc;
      }
      // Each warpgroup reads both accumulators: both groups' last PVs must be complete.  (The same
      // barrier orders every thread's exchange reads before O overwrites the exchange.)
      tc_fence_before();
      named_barrier_sync(kMergeBarrier, 2 * kBlockM);
      tc_fence_after();
      // Each warpgroup normalises half of the head dimension into the staging buffer: row r of
      // 64-column chunk c at kOStOff + c*16 KB + r*128 B, 16-byte units XOR-swizzled by r % 8 (the
      // layout of the O tensor map's 128-byte swizzle).
#pragma unroll
      for (int c = g * (D / 2); c < (g + 1) * (D / 2); c += 32) {
        uint32_t u0[32], u1[32];
        tmem_ld32_nowait(tl + L::kColO + c, u0);
        tmem_ld32_nowait(tl + L::kColO + D + c, u1);
        tmem_wait_ld_regs(u0);
        tmem_wait_ld_regs(u1);
        float o[32];
#pragma unroll
        for (int k2 = 0; k2 < 32; ++k2) {
          o[k2] = fmaf(__uint_as_float(u1[k2]), f1, __uint_as_float(u0[k2]) * f0);
        }
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
      // O_0 and O_1 have been read: the next item's first PVs may overwrite them.
      tc_fence_before();
      mbar_arrive(bar(L::kBarOFree));
      // The staged tile goes out in one TMA store per 64-column chunk (rows past N are clipped);
      // it overlaps the next item.
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

}  // namespace
}  // namespace fa_sm100
