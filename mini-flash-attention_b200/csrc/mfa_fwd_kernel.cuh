// FlashAttention forward for sm_100a: fp16 Q/K/V in [BH, N, 64], fp32 online softmax,
// fp16 output. One CTA owns NQ query tiles of 128 rows of one (batch*head) and streams the
// whole key/value sequence of that head through a TMA + mbarrier ring.
//
// Reference semantics (lavawolfiee/mini-flash-attention):
//   src/mini_flash_attention/flash_attn_cuda.cu:190-368   FlashAttnCuteKernel (per Q tile
//     online softmax over 128-key blocks, P rounded to fp16 for P.V, fp32 row sums)
//   src/mini_flash_attention/flash_attn_cuda.cu:104-169   SoftmaxAccSToPRegs (row max,
//     alpha = e^(m_old - m_new), p = e^(s*scale - m_new), denom = denom*alpha + sum p)
//   src/mini_flash_attention/flash_attn_cuda.cu:73-99     ScaleAccByRow / NormalizeAccByRow
//
// B200 structure (not a translation of the mma.sync kernel):
//   warps 0..8*NQ-1 : softmax warps. Query tile i is owned by warps 8i..8i+7; warp w reads
//                     TMEM lane quadrant w%4 (32 rows, one row per thread) and column half
//                     (w/4)%2 of the tile's 128 scores, so two threads share a row: they trade
//                     their partial row max through shared memory each step and keep partial
//                     row sums that are combined once, in the epilogue.
//   warp  8*NQ      : MMA issuer (whole warp, one elected lane issues): S_i = Q_i K^T (SS
//                     form) and O_i += P_i V (TS form: P straight from TMEM, V consumed
//                     MN-major, so no transpose).
//   warp  8*NQ+1    : TMA producer: Q tiles once, then K and V blocks through STAGES slots.
// TMEM columns: S_i at 128*i, P_i (fp16 pairs) at 128*NQ + 64*i, O_i at 192*NQ + 64*i.
// exp is exp2 with scale*log2(e) folded into one FMA; 3 of every 8 pairs use an FMA-pipe
// polynomial instead of MUFU. The running max is only raised when it grows by more than
// kRescaleThreshold (log2 units), so O is rescaled in TMEM rarely.
// Every mbarrier wait is bounded: on expiry the kernel records a status code, unwinds all
// roles, drains its in-flight copies / MMAs and frees TMEM before returning.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "mfa_exp2.cuh"
#include "mfa_ptx.cuh"

namespace mfa {

struct FwdParams {
  CUtensorMap tm_q;  // [BH][N][64] fp16, box 64 x 128 x 1, 128B swizzle
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  CUtensorMap tm_o;
  int n;                      // sequence length (keys == queries)
  int bh;                     // batch * heads
  int q_blocks;               // ceil(n / (128 * NQ))
  float scale_log2;           // softmax scale * log2(e)
  unsigned long long timeout_ns;  // per-wait watchdog limit
  int* status;                // device status word (0 = ok)
};

// Status codes written to FwdParams::status by the watchdog: kStatusTimeoutBase + site.
constexpr int kStatusTimeoutBase = 0x100;
enum WaitSite : int {
  kSiteLoadKEmpty = 1,
  kSiteLoadVEmpty = 2,
  kSiteMmaQ = 3,
  kSiteMmaK = 4,
  kSiteMmaSFree = 5,
  kSiteMmaV = 6,
  kSiteMmaPFull = 7,
  kSiteSoftSFull = 8,
  kSiteSoftODone = 9,
  kSiteSoftOFinal = 10,
  kSiteSoftExpTok = 11,
};

template <int NQ_, int STAGES_>
struct FwdConfig {
  static constexpr int NQ = NQ_;
  static constexpr int STAGES = STAGES_;
  static constexpr int kRows = 128;       // query rows per tile (= MMA M)
  static constexpr int kKeys = 128;       // keys per block (= S tile N)
  static constexpr int kHeadDim = 64;
  static constexpr int kTileBytes = kRows * kHeadDim * 2;  // 16 KiB, one TMA box
  static constexpr int kSoftmaxWarps = 8 * NQ;   // two warps per TMEM lane quadrant and tile
  static constexpr int kMmaWarp = kSoftmaxWarps;
  static constexpr int kLoadWarp = kSoftmaxWarps + 1;
  // With two query tiles (16 softmax warps) the register file is rebalanced with setmaxnreg,
  // which works per warpgroup: the MMA and TMA warps then fill a fifth warpgroup (2 warps
  // idle). 640 threads launch with 96 registers each (5 warps per SM sub-partition); after
  // the split: 512 x 104 + 128 x 64 = 640 x 96, and per sub-partition 4 x 104 + 64 <= 512.
  static constexpr bool kRebalanceRegs = NQ == 2;
  static constexpr int kThreads = kRebalanceRegs ? 32 * 20 : 32 * (kSoftmaxWarps + 2);
  static constexpr int kLaunchRegs = 96;
  static constexpr int kSoftmaxRegs = 104;
  static constexpr int kControlRegs = 64;

  // shared memory (offsets from a 1024-aligned base; 128B swizzle atoms need 1024 alignment)
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + NQ * kTileBytes;
  static constexpr int kVOff = kKOff + STAGES * kTileBytes;
  static constexpr int kBarOff = kVOff + STAGES * kTileBytes;
  // barrier indices
  static constexpr int kBarQFull = 0;
  static constexpr int kBarKFull = 1;
  static constexpr int kBarKEmpty = kBarKFull + STAGES;
  static constexpr int kBarVFull = kBarKEmpty + STAGES;
  static constexpr int kBarVEmpty = kBarVFull + STAGES;
  static constexpr int kBarSFull = kBarVEmpty + STAGES;
  static constexpr int kBarSFree = kBarSFull + NQ;
  static constexpr int kBarPFull = kBarSFree + NQ;
  static constexpr int kBarODone = kBarPFull + NQ;
  // exp-phase tokens: with two tiles their exp loops take turns (tile 0 first)
  static constexpr int kBarExpTok = kBarODone + NQ;
  static constexpr int kBarDrain = kBarExpTok + 2;
  static constexpr int kNumBars = kBarDrain + 1;
  // partial row max / row sum exchange between the two threads of a row:
  // [step parity][tile][column half][row] floats
  static constexpr int kXchOff = kBarOff + kNumBars * 8;
  static constexpr int kXchBytes = 2 * NQ * 2 * kRows * 4;
  static constexpr int kTmemSlotOff = kXchOff + kXchBytes;
  static constexpr int kAbortOff = kTmemSlotOff + 4;
  static constexpr int kSmemUsed = kAbortOff + 4;
  static constexpr int kSmemBytes = kSmemUsed + 1024;  // slack for manual 1024 alignment

  // tensor memory columns
  static constexpr int kTmemCols = NQ == 2 ? 512 : 256;
  static constexpr int kColS = 0;
  static constexpr int kColP = 128 * NQ;
  static constexpr int kColO = 192 * NQ;

  static constexpr float kRescaleThreshold = 8.0f;
  // exp2 split: pair k of a row uses the polynomial when bit (k % 8) is set (1 of 8 pairs;
  // the polynomial costs ~5 issue slots per element against 1 for MUFU, so a small share
  // relieves MUFU without starving issue).
  static constexpr uint32_t kPolyMask = 0x10u;
  // With two tiles, their exp loops alternate (mbarrier tokens), so one tile's TMEM traffic,
  // max exchange and barrier waits overlap the other tile's MUFU / FMA work.
  static constexpr bool kPingPong = false;
  static_assert(!kRebalanceRegs ||
                    4 * 32 * kSoftmaxRegs * 4 + 4 * 32 * kControlRegs == kThreads * kLaunchRegs,
                "register split must use exactly the launch allocation");
  static_assert(!kRebalanceRegs || 4 * kSoftmaxRegs + kControlRegs <= 512, "per sub-partition");
  static_assert(kColO + 64 * NQ <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct Watchdog {
  volatile int* abort;
  int* status;
  unsigned long long timeout_ns;

  __device__ void trip(int site) const {
    *abort = 1;
    atomicCAS(status, 0, kStatusTimeoutBase + site);
  }
};

// Wait by one thread. Returns false if the CTA is aborting or this wait timed out.
__device__ __forceinline__ bool wait_single(uint32_t bar, uint32_t parity, const Watchdog& wd,
                                            int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 0) {
      if (*wd.abort) return false;
      if (global_timer_ns() - t0 > wd.timeout_ns) {
        wd.trip(site);
        return false;
      }
    }
  }
}

// Warp-collective wait: every lane polls, the warp leaves together with one verdict.
__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, const Watchdog& wd,
                                          int site) {
  const int lane = threadIdx.x & 31;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    const bool ok = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, ok)) return true;
    if ((it & 15u) == 15u) {
      int stop = 0;
      if (lane == 0) {
        if (t0 == 0) t0 = global_timer_ns();
        if (*wd.abort) {
          stop = 1;
        } else if (global_timer_ns() - t0 > wd.timeout_ns) {
          wd.trip(site);
          stop = 1;
        }
      }
      if (__shfl_sync(0xffffffffu, stop, 0)) return false;
    }
  }
}

// Bounded drain used only while unwinding: ignores the abort flag.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > 200000000ull) return;  // 200 ms
  }
}

template <class Cfg>
__device__ __forceinline__ void load_role(const FwdParams& p, uint8_t* smem, uint32_t bars,
                                          int head, int q_row0, int nkb, const Watchdog& wd) {
  constexpr int ST = Cfg::STAGES;
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  const uint32_t sbase = smem_addr(smem);
  tma_prefetch_desc(&p.tm_q);
  tma_prefetch_desc(&p.tm_k);
  tma_prefetch_desc(&p.tm_v);
  tma_prefetch_desc(&p.tm_o);

  mbar_arrive_expect_tx(bar(Cfg::kBarQFull), Cfg::NQ * Cfg::kTileBytes);
#pragma unroll
  for (int i = 0; i < Cfg::NQ; ++i) {
    tma_load_3d(sbase + Cfg::kQOff + i * Cfg::kTileBytes, &p.tm_q, bar(Cfg::kBarQFull), 0,
                q_row0 + i * Cfg::kRows, head);
  }
  // K/V blocks are re-read by every query-tile CTA of this head: keep them in L2.
  const uint64_t keep = l2_policy_evict_last();
  int issued = 0;
  for (int j = 0; j < nkb; ++j) {
    const int st = j % ST;
    const uint32_t ph = static_cast<uint32_t>(j / ST) & 1u;
    if (!wait_single(bar(Cfg::kBarKEmpty + st), ph ^ 1u, wd, kSiteLoadKEmpty)) break;
    mbar_arrive_expect_tx(bar(Cfg::kBarKFull + st), Cfg::kTileBytes);
    tma_load_3d_hint(sbase + Cfg::kKOff + st * Cfg::kTileBytes, &p.tm_k, bar(Cfg::kBarKFull + st),
                     0, j * Cfg::kKeys, head, keep);
    if (!wait_single(bar(Cfg::kBarVEmpty + st), ph ^ 1u, wd, kSiteLoadVEmpty)) {
      issued = -(j + 1);  // K of block j issued, V not
      break;
    }
    mbar_arrive_expect_tx(bar(Cfg::kBarVFull + st), Cfg::kTileBytes);
    tma_load_3d_hint(sbase + Cfg::kVOff + st * Cfg::kTileBytes, &p.tm_v, bar(Cfg::kBarVFull + st),
                     0, j * Cfg::kKeys, head, keep);
    issued = j + 1;
  }
  if (*wd.abort) {
    // Unwinding: wait for every copy this thread put in flight before shared memory goes away.
    drain_wait(bar(Cfg::kBarQFull), 0);
    const int k_blocks = issued >= 0 ? issued : -issued;
    const int v_blocks = issued >= 0 ? issued : -issued - 1;
    for (int st = 0; st < ST; ++st) {
      int last_k = -1, last_v = -1;
      for (int j = st; j < k_blocks; j += ST) last_k = j;
      for (int j = st; j < v_blocks; j += ST) last_v = j;
      if (last_k >= 0) drain_wait(bar(Cfg::kBarKFull + st), static_cast<uint32_t>(last_k / ST) & 1u);
      if (last_v >= 0) drain_wait(bar(Cfg::kBarVFull + st), static_cast<uint32_t>(last_v / ST) & 1u);
    }
  }
}

// Executed by the whole MMA warp: waits and descriptor arithmetic stay warp-uniform (uniform
// datapath, no per-MMA register moves); one elected lane issues tcgen05.mma / commit. Issue
// cost per MMA matters here: a 128x64x16 P.V step is only 32 tensor-core cycles.
template <class Cfg>
__device__ __forceinline__ void mma_role(const FwdParams& p, uint8_t* smem, uint32_t bars,
                                         uint32_t tmem, int nkb, const Watchdog& wd) {
  constexpr int ST = Cfg::STAGES;
  constexpr int NQ = Cfg::NQ;
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  const uint32_t sbase = smem_addr(smem);
  constexpr uint32_t kIdescS = idesc_f16_f32(128, 128, false);
  constexpr uint32_t kIdescO = idesc_f16_f32(128, 64, true);
  // K-major Q / K tiles: SBO = 1024 (8-row swizzle atoms), LBO unused (16).
  constexpr uint32_t kHiKMajor = smem_desc_hi(1024, kSwizzle128B);
  // MN-major V tile (d contiguous): SBO = 1024 between 8-key groups, LBO = one tile (unused,
  // the 64 d-columns are a single 128-byte swizzle atom).
  constexpr uint32_t kHiMNMajor = smem_desc_hi(1024, kSwizzle128B);
  const uint32_t q_lo = smem_desc_lo(sbase + Cfg::kQOff, 16);
  const uint32_t k_lo = smem_desc_lo(sbase + Cfg::kKOff, 16);
  const uint32_t v_lo = smem_desc_lo(sbase + Cfg::kVOff, Cfg::kTileBytes);
  constexpr uint32_t kTileStep = Cfg::kTileBytes >> 4;
  const bool leader = elect_one();
  bool issued_any = false;

  if (!wait_warp(bar(Cfg::kBarQFull), 0, wd, kSiteMmaQ)) goto unwind;

  for (int j = -1; j < nkb; ++j) {
    // ---- S_i[j+1] = Q_i K_{j+1}^T as soon as softmax_i has pulled S_i[j] into registers.
    if (j + 1 < nkb) {
      const int st1 = (j + 1) % ST;
      const uint32_t ph1 = static_cast<uint32_t>((j + 1) / ST) & 1u;
      if (!wait_warp(bar(Cfg::kBarKFull + st1), ph1, wd, kSiteMmaK)) goto unwind;
      const uint32_t kd = k_lo + st1 * kTileStep;
#pragma unroll
      for (int i = 0; i < NQ; ++i) {
        if (j >= 0) {
          if (!wait_warp(bar(Cfg::kBarSFree + i), static_cast<uint32_t>(j) & 1u, wd,
                         kSiteMmaSFree))
            goto unwind;
        }
        tc_fence_after();
        if (leader) {
          const uint32_t qd = q_lo + i * kTileStep;
          const uint32_t d_tmem = tmem + Cfg::kColS + 128 * i;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // 16 of the 64 head dims per MMA (32 bytes)
            mma_ss(d_tmem, desc_join(qd + 2 * kk, kHiKMajor), desc_join(kd + 2 * kk, kHiKMajor),
                   kIdescS, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar(Cfg::kBarSFull + i));
        }
        __syncwarp();
        issued_any = true;
      }
      if (leader) mma_commit(bar(Cfg::kBarKEmpty + st1));
      __syncwarp();
    }
    if (j < 0) continue;
    // ---- O_i += P_i[j] V_j once softmax_i has written P_i[j] (and rescaled O_i if needed).
    const int st = j % ST;
    const uint32_t ph = static_cast<uint32_t>(j / ST) & 1u;
    if (!wait_warp(bar(Cfg::kBarVFull + st), ph, wd, kSiteMmaV)) goto unwind;
    const uint32_t vd = v_lo + st * kTileStep;
#pragma unroll
    for (int i = 0; i < NQ; ++i) {
      if (!wait_warp(bar(Cfg::kBarPFull + i), static_cast<uint32_t>(j) & 1u, wd, kSiteMmaPFull))
        goto unwind;
      tc_fence_after();
      if (leader) {
        const uint32_t d_tmem = tmem + Cfg::kColO + 64 * i;
        const uint32_t a_tmem = tmem + Cfg::kColP + 64 * i;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // 16 keys per MMA: two 8-key swizzle atoms (2 KiB)
          mma_ts(d_tmem, a_tmem + 8 * kk, desc_join(vd + 128 * kk, kHiMNMajor), kIdescO,
                 (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar(Cfg::kBarODone + i));
      }
      __syncwarp();
      issued_any = true;
    }
    if (leader) mma_commit(bar(Cfg::kBarVEmpty + st));
    __syncwarp();
  }
  return;

unwind:
  if (issued_any) {
    // Let every MMA this warp issued finish before TMEM is released.
    if (leader) mma_commit(bar(Cfg::kBarDrain));
    __syncwarp();
    drain_wait(bar(Cfg::kBarDrain), 0);
  }
}

template <class Cfg>
__device__ __forceinline__ void softmax_role(const FwdParams& p, uint8_t* smem, uint32_t bars,
                                             uint32_t tmem, int tile, int head, int q_row0,
                                             int nkb, const Watchdog& wd) {
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quad = warp & 3;              // TMEM lane quadrant this warp may access
  const int half = (warp >> 2) & 1;       // which 64 of the tile's 128 key columns
  const int row = quad * 32 + lane;       // row of the query tile == TMEM lane
  const uint32_t lane_bits = static_cast<uint32_t>(quad * 32) << 16;
  const uint32_t tS = tmem + lane_bits + Cfg::kColS + 128 * tile + 64 * half;
  const uint32_t tP = tmem + lane_bits + Cfg::kColP + 64 * tile + 32 * half;
  const uint32_t tO = tmem + lane_bits + Cfg::kColO + 64 * tile + 32 * half;
  // partner exchange slots: xch[parity][tile][half][row]
  float* xch = reinterpret_cast<float*>(smem + Cfg::kXchOff);
  auto slot = [&](int parity, int h) {
    return xch + ((parity * Cfg::NQ + tile) * 2 + h) * Cfg::kRows + row;
  };
  const int pair_bar = 1 + tile * 4 + quad;  // the two warps that share these 32 rows
  const float c = p.scale_log2;

  float m_run = -INFINITY;  // running max of s*scale*log2(e), identical in both threads
  float l_run = 0.0f;       // this thread's partial sum of p over its column half
  bool ok = true;
  // Tile 1 hands tile 0 the first exp turn.
  if (Cfg::kPingPong && tile == 1 && lane == 0) mbar_arrive(bar(Cfg::kBarExpTok + 0));

  for (int j = 0; j < nkb; ++j) {
    if (!wait_warp(bar(Cfg::kBarSFull + tile), static_cast<uint32_t>(j) & 1u, wd, kSiteSoftSFull)) {
      ok = false;
      break;
    }
    tc_fence_after();
    uint32_t sr[64];
    tmem_ld64_sync(tS, sr);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(Cfg::kBarSFree + tile));

    const int valid = p.n - j * Cfg::kKeys - 64 * half;
    if (valid < 64) {
#pragma unroll
      for (int k = 0; k < 64; ++k)
        if (k >= valid) sr[k] = __float_as_uint(-INFINITY);
    }

    // Partial max over this half: four 3-input max chains (4 seeds, 7 x 8, 4 tail = 64).
    float mx[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) mx[a] = __uint_as_float(sr[a]);
#pragma unroll
    for (int k = 4; k < 60; k += 8) {
#pragma unroll
      for (int a = 0; a < 4; ++a)
        mx[a] = max3(mx[a], __uint_as_float(sr[k + 2 * a]), __uint_as_float(sr[k + 2 * a + 1]));
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) mx[a] = fmaxf(mx[a], __uint_as_float(sr[60 + a]));
    const float pm = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
    // Trade partial maxima with the partner thread (same row, other half). Slots alternate
    // with the step parity so a partner one step ahead never overwrites an unread value.
    *slot(j & 1, half) = pm;
    named_bar_sync(pair_bar, 64);
    const float m_blk = fmaxf(pm, *slot(j & 1, half ^ 1)) * c;
    const float m_new = fmaxf(m_run, m_blk);
    // Raise the reference max only when some row of the warp grew past the threshold. Both
    // warps of a pair hold the same rows and values, so they take the same decision.
    const bool grow = __any_sync(0xffffffffu, m_new > m_run + Cfg::kRescaleThreshold);
    const float m_use = grow ? m_new : m_run;
    const float alpha = ex2_approx(m_run - m_use);  // 0 on the first block (m_run = -inf)
    float neg_m = -m_use;
    if constexpr (Cfg::kPingPong) {
      if (!wait_warp(bar(Cfg::kBarExpTok + tile), static_cast<uint32_t>(j) & 1u, wd,
                     kSiteSoftExpTok)) {
        ok = false;
        break;
      }
      // Pin the exp loop below the token wait: it depends on neg_m "produced" here.
      asm volatile("" : "+f"(neg_m)::"memory");
    }

    // Scale-subtract and row sum run on packed pairs (fma/add .f32x2). Pairs whose index
    // has its bit set in kPolyMask take exp2 from the FMA-pipe polynomial, the others from
    // MUFU ex2, so both units work on every row.
    const uint64_t c2 = f2_splat(c);
    const uint64_t negm2 = f2_splat(neg_m);
    uint32_t pk[32];
    uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const uint64_t x =
          f2_fma(f2_pack(__uint_as_float(sr[2 * k]), __uint_as_float(sr[2 * k + 1])), c2, negm2);
      float x0, x1, e0, e1;
      f2_unpack(x, x0, x1);
      if ((Cfg::kPolyMask >> (k & 7)) & 1u) {
        exp2_poly_pair(x0, x1, e0, e1);
      } else {
        e0 = ex2_approx(x0);
        e1 = ex2_approx(x1);
      }
      acc[k & 3] = f2_add(acc[k & 3], f2_pack(e0, e1));
      pk[k] = pack_half2(e0, e1);
    }
    float acc0, acc1, acc2, acc3;
    f2_unpack(f2_add(acc[0], acc[1]), acc0, acc1);
    f2_unpack(f2_add(acc[2], acc[3]), acc2, acc3);
    l_run = l_run * alpha + ((acc0 + acc1) + (acc2 + acc3));
    m_run = m_use;
    if constexpr (Cfg::kPingPong) {
      // Keep the exp results above the hand-over, then pass the turn to the other tile.
      regs_ready(pk, l_run);
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(Cfg::kBarExpTok + (tile ^ 1)));
    }

    // P_i and O_i are free once the previous O_i += P_i V has completed.
    if (j > 0) {
      if (!wait_warp(bar(Cfg::kBarODone + tile), static_cast<uint32_t>(j - 1) & 1u, wd,
                     kSiteSoftODone)) {
        ok = false;
        break;
      }
      tc_fence_after();
    }
    tmem_st32(tP, pk);
    if (grow && j > 0) {
      uint32_t o[32];
      tmem_ld32_sync(tO, o);
#pragma unroll
      for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
      tmem_st32(tO, o);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(Cfg::kBarPFull + tile));
  }

  // ---- epilogue: O / l -> fp16 -> swizzled staging (this tile's Q slot) -> TMA store.
  if (ok) {
    ok = wait_warp(bar(Cfg::kBarODone + tile), static_cast<uint32_t>(nkb - 1) & 1u, wd,
                   kSiteSoftOFinal);
  }
  // Row sum = both halves' partial sums (every thread reaches this barrier, ok or not).
  *slot(nkb & 1, half) = l_run;
  named_bar_sync(pair_bar, 64);
  const float l_row = l_run + *slot(nkb & 1, half ^ 1);
  uint8_t* stage = smem + Cfg::kQOff + tile * Cfg::kTileBytes;
  if (ok) {
    tc_fence_after();
    const float inv_l = 1.0f / l_row;
    uint32_t o[32];
    tmem_ld32_sync(tO, o);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {  // 4 chunks of 8 halves = 16 bytes each
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        w[e] = pack_half2(__uint_as_float(o[8 * ch + 2 * e]) * inv_l,
                          __uint_as_float(o[8 * ch + 2 * e + 1]) * inv_l);
      }
      const int chunk = 4 * half + ch;
      const uint32_t dst = smem_addr(stage + row * 128 + ((chunk ^ (row & 7)) << 4));
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w[0]), "r"(w[1]),
                   "r"(w[2]), "r"(w[3])
                   : "memory");
    }
    fence_proxy_async_smem();
  }
  named_bar_sync(9 + tile, 256);
  if (ok && half == 0 && row == 0 && !*wd.abort) {
    const int r0 = q_row0 + tile * Cfg::kRows;
    if (r0 < p.n) {
      tma_store_3d(&p.tm_o, smem_addr(stage), 0, r0, head);
      tma_store_commit();
      tma_store_wait_read();
    }
  }
}

template <int NQ, int STAGES>
__global__ void __launch_bounds__(FwdConfig<NQ, STAGES>::kThreads, 1)
    mfa_fwd_kernel(const __grid_constant__ FwdParams p) {
  using Cfg = FwdConfig<NQ, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = static_cast<int>(blockIdx.x) / p.q_blocks;
  const int q_block = static_cast<int>(blockIdx.x) % p.q_blocks;
  const int q_row0 = q_block * Cfg::kRows * NQ;
  const int nkb = (p.n + Cfg::kKeys - 1) / Cfg::kKeys;

  const uint32_t bars = smem_addr(smem + Cfg::kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kTmemSlotOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kAbortOff);

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(bars + 8 * Cfg::kBarQFull, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bars + 8 * (Cfg::kBarKFull + s), 1);
      mbar_init(bars + 8 * (Cfg::kBarKEmpty + s), 1);
      mbar_init(bars + 8 * (Cfg::kBarVFull + s), 1);
      mbar_init(bars + 8 * (Cfg::kBarVEmpty + s), 1);
    }
    for (int i = 0; i < NQ; ++i) {
      mbar_init(bars + 8 * (Cfg::kBarSFull + i), 1);
      mbar_init(bars + 8 * (Cfg::kBarSFree + i), 8);  // one arrive per softmax warp of tile i
      mbar_init(bars + 8 * (Cfg::kBarPFull + i), 8);
      mbar_init(bars + 8 * (Cfg::kBarODone + i), 1);
    }
    mbar_init(bars + 8 * (Cfg::kBarExpTok + 0), 8);
    mbar_init(bars + 8 * (Cfg::kBarExpTok + 1), 8);
    mbar_init(bars + 8 * Cfg::kBarDrain, 1);
    mbar_init_fence();
  }
  if (warp == 0) {
    tmem_alloc(smem_addr(tmem_slot), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Watchdog wd{abort_flag, p.status, p.timeout_ns};

  if (warp >= Cfg::kSoftmaxWarps) {
    if constexpr (Cfg::kRebalanceRegs) setmaxnreg_dec<Cfg::kControlRegs>();
    if (warp == Cfg::kLoadWarp) {
      if (lane == 0) load_role<Cfg>(p, smem, bars, head, q_row0, nkb, wd);
    } else if (warp == Cfg::kMmaWarp) {
      mma_role<Cfg>(p, smem, bars, tmem, nkb, wd);
    }
  } else {
    if constexpr (Cfg::kRebalanceRegs) setmaxnreg_inc<Cfg::kSoftmaxRegs>();
    softmax_role<Cfg>(p, smem, bars, tmem, warp / 8, head, q_row0, nkb, wd);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace mfa
