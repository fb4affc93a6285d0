// FlashAttention forward for sm_100a: fp16 Q/K/V in [BH, N, 64], fp32 online softmax,
// fp16 output. Persistent: one CTA per SM walks a contiguous range of work units
// (head, query block of 128*NQ rows, key block of 128 keys) and streams K/V through a TMA +
// mbarrier ring that runs across unit boundaries.
//
// Reference semantics (lavawolfiee/mini-flash-attention):
//   src/mini_flash_attention/flash_attn_cuda.cu:190-368   FlashAttnCuteKernel (per Q tile
//     online softmax over 128-key blocks, P rounded to fp16 for P.V, fp32 row sums)
//   src/mini_flash_attention/flash_attn_cuda.cu:104-169   SoftmaxAccSToPRegs (row max,
//     alpha = e^(m_old - m_new), p = e^(s*scale - m_new), denom = denom*alpha + sum p)
//   src/mini_flash_attention/flash_attn_cuda.cu:73-99     ScaleAccByRow / NormalizeAccByRow
//
// B200 structure (not a translation of the mma.sync kernel):
//   warps 0..8*NQ-1 : softmax warps. With two tiles, tile i is owned by warps 4i..4i+3 (upper
//                     halves of the four TMEM lane quadrants) and 8+4i..8+4i+3 (lower halves),
//                     so each sub-partition holds one warp of each tile in its first two and
//                     its last two warp slots; with one tile, warps 0..7. Warp w reads
//                     16 rows of TMEM lane quadrant w%4 (upper or lower half) as
//                     16x256b fragments: four neighbouring lanes share a row, two of every
//                     eight columns each, so row maxima and sums are warp shuffles and the
//                     softmax warps never wait for one another.
//   warp  8*NQ      : MMA issuer (whole warp, one elected lane issues): S_i = Q_i K^T (SS
//                     form) and O_i += P_i V (TS form: P straight from TMEM, V consumed
//                     MN-major, so no transpose). With two query tiles it issues tile 0's
//                     products and warp 8*NQ+3 issues tile 1's: one thread issues a
//                     tcgen05.mma about every 60-70 cycles, more than a 128x64x16 P.V
//                     product takes on the tensor core (32 cycles), so a single issuer
//                     cannot keep the tensor core busy (measured: the same MMA stream with
//                     no softmax in the way runs 1.29x faster from two warps).
//   warp  8*NQ+1    : TMA producer: the Q tiles of each unit (two Q buffers, so the next
//                     unit's Q loads while this one runs), then K and V blocks.
//   warp  8*NQ+2    : (NQ = 2) TMA stores of finished units' output (staged in their Q
//                     buffer), so the softmax warps go on to the next unit without waiting.
// TMEM columns: S_i at 128*i, P_i (fp16 pairs) at 128*NQ + 64*i, O_i at 192*NQ + 64*i.
// exp is exp2 with scale*log2(e) folded into one FMA; 1 of every 8 pairs uses an FMA-pipe
// polynomial instead of MUFU. The running max is only raised when it grows by more than
// kRescaleThreshold (log2 units), so O is rescaled in TMEM rarely.
// Work split: see FwdParams::split. A unit range that covers a whole query block ends with
// O / l stored as fp16 by TMA; a piece of a query block leaves fp32 partial results in the
// workspace for mfa_merge_kernel.
// Every mbarrier wait is bounded: on expiry the kernel records a status code, unwinds all
// roles, drains its in-flight copies / MMAs and frees TMEM before returning.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "mfa_common.cuh"
#include "mfa_exp2.cuh"
#include "mfa_ptx.cuh"
#include "mfa_schedule.cuh"

namespace mfa {

template <int NQ_, int STAGES_, bool CAUSAL_, bool BF16_, int D_, bool LSE_ = false>
struct FwdConfig {
  static constexpr bool kLSE = LSE_;  // also write the row log-sum-exp (FwdParams::lse)
  static constexpr int NQ = NQ_;
  static constexpr int STAGES = STAGES_;
  static constexpr bool kCausal = CAUSAL_;  // mask key index > query index
  static constexpr bool kBF16 = BF16_;      // q, k, v, P and out in bf16 instead of fp16
  static constexpr int kRows = 128;       // query rows per tile (= MMA M)
  static constexpr int kRowsPerUnit = kRows * NQ;
  static constexpr int kKeys = 128;       // keys per block (= S tile N)
  static constexpr int kHeadDim = D_;     // 32, 64 or 128
  static constexpr int kTileBytes = kRows * kHeadDim * 2;  // one 128-row tile of q, k or v
  // A tile arrives as D / 64 TMA boxes of 64 columns (128-byte rows, 128-byte swizzle), or
  // for D = 32 as one box of 32 columns (64-byte rows, 64-byte swizzle); boxes are stored
  // one after the other. The MMA operand descriptors follow the same atoms.
  static constexpr int kBoxCols = kHeadDim < 64 ? kHeadDim : 64;
  static constexpr int kBoxes = kHeadDim / kBoxCols;
  static constexpr int kRowBytes = kBoxCols * 2;          // bytes of one box row = swizzle span
  static constexpr int kBoxBytes = kRows * kRowBytes;
  static constexpr int kSwizzleChunks = kRowBytes / 16;   // 16-byte chunks per swizzled row
  static constexpr int kSoftmaxWarps = 8 * NQ;   // two warps per TMEM lane quadrant and tile
  static constexpr int kMmaWarp = kSoftmaxWarps;
  static constexpr int kLoadWarp = kSoftmaxWarps + 1;
  // Output stores of finished units: a store warp with two query tiles (in the fifth
  // warpgroup); with one tile the first softmax warp of the tile issues them
  // (a third non-softmax warp next to two softmax warps per sub-partition measured slower).
  static constexpr bool kStoreRole = NQ == 2;
  static constexpr int kStoreWarp = kSoftmaxWarps + 2;
  // MMA issuers: one per query tile (tile 1's is the fifth warpgroup's fourth warp). Each
  // commits once per step on the K / V empty barriers, which therefore count NQ arrivals.
  static constexpr int kMmaWarp2 = kSoftmaxWarps + 3;
  // With two query tiles (16 softmax warps) the register file is rebalanced with setmaxnreg,
  // which works per warpgroup: the two MMA warps, the load and the store warp then fill a
  // fifth warpgroup. 640 threads launch with 96 registers each (5 warps per SM
  // sub-partition); after the split: 512 x 104 + 128 x 64 = 640 x 96, and per sub-partition
  // 4 x 104 + 64 <= 512.
  static constexpr bool kRebalanceRegs = NQ == 2;
  static constexpr int kThreads = kRebalanceRegs ? 32 * 20 : 32 * (kSoftmaxWarps + 2);
  static constexpr int kLaunchRegs = 96;
  static constexpr int kSoftmaxRegs = 104;
  static constexpr int kControlRegs = 64;

  // shared memory (offsets from a 1024-aligned base; swizzle atoms need 1024 / 512 alignment)
  static constexpr int kQOff = 0;                              // two Q buffers of NQ tiles
  static constexpr int kKOff = kQOff + 2 * NQ * kTileBytes;
  static constexpr int kVOff = kKOff + STAGES * kTileBytes;
  static constexpr int kBarOff = kVOff + STAGES * kTileBytes;
  // barrier indices
  static constexpr int kBarQFull = 0;                 // [2]
  static constexpr int kBarQEmpty = 2;                // [2]
  static constexpr int kBarKFull = 4;
  static constexpr int kBarKEmpty = kBarKFull + STAGES;
  static constexpr int kBarVFull = kBarKEmpty + STAGES;
  static constexpr int kBarVEmpty = kBarVFull + STAGES;
  static constexpr int kBarSFull = kBarVEmpty + STAGES;
  static constexpr int kBarSFree = kBarSFull + NQ;
  static constexpr int kBarPFull = kBarSFree + NQ;
  static constexpr int kBarODone = kBarPFull + NQ;
  static constexpr int kBarStage = kBarODone + NQ;  // [tile]: output staging written
  static constexpr int kBarDrain = kBarStage + NQ;  // [NQ]: one per MMA warp
  static constexpr int kNumBars = kBarDrain + NQ;
  static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr int kAbortOff = kTmemSlotOff + 4;
  static constexpr int kSmemUsed = kAbortOff + 4;
  static constexpr int kSmemBytes = kSmemUsed + 1024;  // slack for manual 1024 alignment

  // tensor memory columns: S_i (128 fp32), P_i (64 fp16 pairs), O_i (D fp32)
  static constexpr int kColS = 0;
  static constexpr int kColP = 128 * NQ;
  static constexpr int kColO = 192 * NQ;
  static constexpr int kTmemUsed = kColO + kHeadDim * NQ;
  static constexpr int kTmemCols = kTmemUsed <= 256 ? 256 : 512;  // allocation: a power of 2

  // one partial-result slot: O[rows][D] fp32 (unnormalised), then m[rows], l[rows]
  static constexpr int kSlotFloats = kRowsPerUnit * (kHeadDim + 2);

  static constexpr float kRescaleThreshold = 8.0f;
  // exp2 split: pair k of a row uses the polynomial when bit (k % 8) is set (1 of 8 pairs;
  // the polynomial costs ~5 issue slots per element against 1 for MUFU, so a small share
  // relieves MUFU without starving issue).
  static constexpr uint32_t kPolyMask = 0x10u;

  static_assert(!kRebalanceRegs ||
                    4 * 32 * kSoftmaxRegs * 4 + 4 * 32 * kControlRegs == kThreads * kLaunchRegs,
                "register split must use exactly the launch allocation");
  static_assert(!kRebalanceRegs || 4 * kSoftmaxRegs + kControlRegs <= 512, "per sub-partition");
  static_assert(kTmemUsed <= 512, "TMEM budget");
  static_assert(kHeadDim == 32 || kHeadDim == 64 || kHeadDim == 128, "head dim");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// ---------------------------------------------------------------- unit schedule
// Walks the steps (one key block of one query block each) of this CTA's work in order. Two
// orders, chosen by FwdParams::split:
//   split == 0: whole query blocks u = cta, cta + ctas, cta + 2 ctas, ... so that the CTAs
//               running at the same time work on neighbouring query blocks, mostly of the
//               same head, and its K/V blocks are read from L2 by all of them;
//   split == 1: the contiguous step range split_range() (a head's K/V then fits in L2 anyway:
//               split mode is chosen when there are few query blocks, or with causal masking,
//               whose query blocks differ in length).
// Six 32-bit words of state: it is live across the softmax loop, where registers are scarce
// (the launcher guarantees fewer than 2^31 units and steps per CTA). In split mode only the
// range's first segment can start inside a query block and only its last can stop inside one.
template <bool kCausal>
struct StepCursor {
  int u;        // current query block, row-major over (head, query block)
  int j;        // current key block
  int j0, j1;   // key blocks [j0, j1) of u handled in this segment
  int rem;      // split: steps after this segment; whole blocks: query blocks after this one
  int seg_idx;  // index of the current segment

  __device__ void init(const FwdParams& p) {
    const Schedule& sc = p.sc;
    const long long units = static_cast<long long>(sc.bh) * sc.q_blocks;
    seg_idx = 0;
    if (!p.split) {
      u = static_cast<int>(blockIdx.x);
      j = j0 = 0;
      j1 = u < units ? sc.nkb : 0;
      rem = u < units ? static_cast<int>((units - 1 - u) / gridDim.x) : 0;
      return;
    }
    long long b, e;
    sc.range(static_cast<int>(blockIdx.x), b, e);  // gridDim.x == sc.ctas
    if (b >= e) {
      u = j = j0 = j1 = rem = 0;
      return;
    }
    sc.locate<kCausal>(b, u, j0);
    j = j0;
    const long long len = e - b;
    const int avail = sc.steps_of<kCausal>(sc.qb_of(u)) - j0;
    j1 = len < avail ? j0 + static_cast<int>(len) : j0 + avail;
    rem = static_cast<int>(len - (j1 - j0));
  }
  __device__ bool valid() const { return j < j1; }
  __device__ bool first_step() const { return j == j0; }
  __device__ bool first_of_range() const { return seg_idx == 0; }
  __device__ bool whole(const Schedule& sc) const {
    return j0 == 0 && j1 == sc.steps_of<kCausal>(sc.qb_of(u));
  }
  // Advance to the next segment (the softmax warps walk a segment with their own counter).
  __device__ void next_segment(const FwdParams& p) {
    j = j1 - 1;
    step(p);
  }
  __device__ void step(const FwdParams& p) {
    if (++j >= j1 && rem > 0) {
      if (p.split) {
        u = p.sc.next_unit<kCausal>(u);
        const int steps = p.sc.steps_of<kCausal>(p.sc.qb_of(u));
        j1 = rem < steps ? rem : steps;
        rem -= j1;
      } else {
        u += static_cast<int>(gridDim.x);
        j1 = p.sc.nkb;
        --rem;
      }
      j = j0 = 0;
      ++seg_idx;
    }
  }
};

// Head and batch index of unit u: its (batch * head) row is u / q_blocks, heads fastest.
__device__ __forceinline__ HeadBatch head_batch(const FwdParams& p, int u) {
  const int bh = p.sc.head_of(u);
  return {bh % p.heads, bh / p.heads};
}

template <class Cfg>
__device__ __forceinline__ void load_role(const FwdParams& p, uint8_t* smem, uint32_t bars,
                                          const Watchdog& wd) {
  constexpr int ST = Cfg::STAGES;
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  const uint32_t sbase = smem_addr(smem);
  tma_prefetch_desc(&p.tm_q);
  tma_prefetch_desc(&p.tm_k);
  tma_prefetch_desc(&p.tm_v);
  tma_prefetch_desc(&p.tm_o);
  // K/V blocks are re-read by every query-block pass over the same head: keep them in L2.
  const uint64_t keep = l2_policy_evict_last();

  StepCursor<Cfg::kCausal> cur;
  cur.init(p);
  int g = 0;  // global step index of this CTA
  int q_loaded = 0, k_issued = 0, v_issued = 0;
  HeadBatch hb = head_batch(p, cur.u);
  while (cur.valid()) {
    if (cur.first_step()) {
      hb = head_batch(p, cur.u);
      const int s = cur.seg_idx, b = s & 1;
      if (!wait_single(bar(Cfg::kBarQEmpty + b), (static_cast<uint32_t>(s >> 1) & 1u) ^ 1u, wd,
                       kSiteLoadQEmpty))
        break;
      mbar_arrive_expect_tx(bar(Cfg::kBarQFull + b), Cfg::NQ * Cfg::kTileBytes);
#pragma unroll
      for (int i = 0; i < Cfg::NQ; ++i) {
#pragma unroll
        for (int x = 0; x < Cfg::kBoxes; ++x) {
          tma_load_4d(sbase + Cfg::kQOff + (b * Cfg::NQ + i) * Cfg::kTileBytes + x * Cfg::kBoxBytes,
                      &p.tm_q, bar(Cfg::kBarQFull + b), x * Cfg::kBoxCols,
                      p.sc.qb_of(cur.u) * Cfg::kRowsPerUnit + i * Cfg::kRows, hb.h, hb.b);
        }
      }
      q_loaded = s + 1;
    }
    const int st = g % ST;
    const uint32_t ph = static_cast<uint32_t>(g / ST) & 1u;
    if (!wait_single(bar(Cfg::kBarKEmpty + st), ph ^ 1u, wd, kSiteLoadKEmpty)) break;
    mbar_arrive_expect_tx(bar(Cfg::kBarKFull + st), Cfg::kTileBytes);
#pragma unroll
    for (int x = 0; x < Cfg::kBoxes; ++x) {
      tma_load_4d_hint(sbase + Cfg::kKOff + st * Cfg::kTileBytes + x * Cfg::kBoxBytes, &p.tm_k,
                       bar(Cfg::kBarKFull + st), x * Cfg::kBoxCols, cur.j * Cfg::kKeys, hb.h,
                       hb.b, keep);
    }
    k_issued = g + 1;
    if (!wait_single(bar(Cfg::kBarVEmpty + st), ph ^ 1u, wd, kSiteLoadVEmpty)) break;
    mbar_arrive_expect_tx(bar(Cfg::kBarVFull + st), Cfg::kTileBytes);
#pragma unroll
    for (int x = 0; x < Cfg::kBoxes; ++x) {
      tma_load_4d_hint(sbase + Cfg::kVOff + st * Cfg::kTileBytes + x * Cfg::kBoxBytes, &p.tm_v,
                       bar(Cfg::kBarVFull + st), x * Cfg::kBoxCols, cur.j * Cfg::kKeys, hb.h,
                       hb.b, keep);
    }
    v_issued = g + 1;
    ++g;
    cur.step(p);
  }
  if (*wd.abort) {
    // Unwinding: wait for every copy this thread put in flight before shared memory goes away.
    for (int b = 0; b < 2; ++b) {
      int last = -1;
      for (int s = b; s < q_loaded; s += 2) last = s;
      if (last >= 0) drain_wait(bar(Cfg::kBarQFull + b), static_cast<uint32_t>(last >> 1) & 1u);
    }
    for (int st = 0; st < ST; ++st) {
      int last_k = -1, last_v = -1;
      for (int x = st; x < k_issued; x += ST) last_k = x;
      for (int x = st; x < v_issued; x += ST) last_v = x;
      if (last_k >= 0) drain_wait(bar(Cfg::kBarKFull + st), static_cast<uint32_t>(last_k / ST) & 1u);
      if (last_v >= 0) drain_wait(bar(Cfg::kBarVFull + st), static_cast<uint32_t>(last_v / ST) & 1u);
    }
  }
}

// Executed by the whole MMA warp: waits and descriptor arithmetic stay warp-uniform (uniform
// datapath, no per-MMA register moves); one elected lane issues tcgen05.mma / commit. Issue
// cost per MMA matters here: a 128x64x16 P.V step is only 32 tensor-core cycles. S for step
// g+1 is issued before P.V of step g, so the next scores are computed while the softmax warps
// still work on the current block (also across unit boundaries). Each MMA warp issues the
// products of one query tile, so each tile's products follow its own softmax warps and no tile
// waits for the other's P.
template <class Cfg>
__device__ __forceinline__ void mma_role(const FwdParams& p, uint8_t* smem, uint32_t bars,
                                         uint32_t tmem, const Watchdog& wd, int tile) {
  constexpr int ST = Cfg::STAGES;
  constexpr int NQ = Cfg::NQ;
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  const uint32_t sbase = smem_addr(smem);
  constexpr uint32_t kIdescS = idesc_f16_f32(128, 128, false, Cfg::kBF16);
  constexpr uint32_t kIdescO = idesc_f16_f32(128, Cfg::kHeadDim, true, Cfg::kBF16);
  // Swizzle atoms are 8 rows of kRowBytes (128 B, or 64 B for D = 32). K-major Q / K tiles:
  // SBO = one atom (8 rows), LBO unused (16); the K steps of 16 head dims (32 bytes) walk
  // through an atom and then on to the next box. MN-major V tile (d contiguous): SBO = one
  // atom between 8-key groups, LBO = one box between the 64-column halves of D = 128 (unused
  // when D fits one atom).
  constexpr uint64_t kSwz = Cfg::kRowBytes == 128 ? kSwizzle128B : kSwizzle64B;
  constexpr uint32_t kHi = smem_desc_hi(8 * Cfg::kRowBytes, kSwz);
  const uint32_t q_lo = smem_desc_lo(sbase + Cfg::kQOff, 16);
  const uint32_t k_lo = smem_desc_lo(sbase + Cfg::kKOff, 16);
  const uint32_t v_lo = smem_desc_lo(sbase + Cfg::kVOff, Cfg::kBoxBytes);
  constexpr uint32_t kTileStep = Cfg::kTileBytes >> 4;
  constexpr int kStepsPerBox = Cfg::kBoxCols / 16;
  // descriptor offset (16-byte units) of K step kk of a K-major tile
  auto k_off = [](int kk) -> uint32_t {
    return static_cast<uint32_t>((kk / kStepsPerBox) * (Cfg::kBoxBytes >> 4) +
                                 (kk % kStepsPerBox) * 2);
  };
  const bool leader = elect_one();
  bool issued_any = false;

  StepCursor<Cfg::kCausal> cs, cp;  // next S step, next P.V step
  cs.init(p);
  cp.init(p);
  int gs = 0, gp = 0;
  // S_i[gs] = Q_i K_gs^T once softmax_i has pulled S_i[gs-1] into registers.
  auto issue_s = [&]() -> bool {
    const int b = cs.seg_idx & 1;
    if (cs.first_step()) {
      if (!wait_warp(bar(Cfg::kBarQFull + b), static_cast<uint32_t>(cs.seg_idx >> 1) & 1u, wd,
                     kSiteMmaQ))
        return false;
    }
    const int st = gs % ST;
    if (!wait_warp(bar(Cfg::kBarKFull + st), static_cast<uint32_t>(gs / ST) & 1u, wd, kSiteMmaK))
      return false;
    const uint32_t kd = k_lo + st * kTileStep;
    {
      const int i = tile;
      if (gs > 0) {
        if (!wait_warp(bar(Cfg::kBarSFree + i), static_cast<uint32_t>(gs - 1) & 1u, wd,
                       kSiteMmaSFree))
          return false;
      }
      tc_fence_after();
      if (leader) {
        const uint32_t qd = q_lo + (b * NQ + i) * kTileStep;
        const uint32_t d_tmem = tmem + Cfg::kColS + 128 * i;
#pragma unroll
        for (int kk = 0; kk < Cfg::kHeadDim / 16; ++kk) {  // 16 head dims per MMA (32 bytes)
          mma_ss(d_tmem, desc_join(qd + k_off(kk), kHi), desc_join(kd + k_off(kk), kHi),
                 kIdescS, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar(Cfg::kBarSFull + i));
      }
      __syncwarp();
      issued_any = true;
    }
    if (leader) mma_commit(bar(Cfg::kBarKEmpty + st));
    __syncwarp();
    ++gs;
    cs.step(p);
    return true;
  };

  if (cs.valid() && !issue_s()) goto unwind;
  while (cp.valid()) {
    // S of the next step goes in before P.V of this one, so the tensor core computes the
    // next scores while the softmax warps are still busy with this block.
    if (cs.valid() && !issue_s()) goto unwind;
    // ---- O_i += P_i[gp] V_gp once softmax_i has written P_i[gp] (and rescaled O_i if needed).
    {
      const int st = gp % ST;
      if (!wait_warp(bar(Cfg::kBarVFull + st), static_cast<uint32_t>(gp / ST) & 1u, wd, kSiteMmaV))
        goto unwind;
      const uint32_t vd = v_lo + st * kTileStep;
      const bool fresh = cp.first_step();  // first block of a unit: overwrite O
      {
        const int i = tile;
        if (!wait_warp(bar(Cfg::kBarPFull + i), static_cast<uint32_t>(gp) & 1u, wd,
                       kSiteMmaPFull))
          goto unwind;
        tc_fence_after();
        if (leader) {
          const uint32_t d_tmem = tmem + Cfg::kColO + Cfg::kHeadDim * i;
          const uint32_t a_tmem = tmem + Cfg::kColP + 64 * i;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {  // 16 keys per MMA: two 8-key swizzle atoms
            mma_ts(d_tmem, a_tmem + 8 * kk, desc_join(vd + Cfg::kRowBytes * kk, kHi), kIdescO,
                   (!fresh || kk > 0) ? 1u : 0u);
          }
          mma_commit(bar(Cfg::kBarODone + i));
        }
        __syncwarp();
        issued_any = true;
      }
      if (leader) mma_commit(bar(Cfg::kBarVEmpty + st));
      __syncwarp();
      ++gp;
      cp.step(p);
    }
  }
  return;

unwind:
  if (issued_any) {
    // Let every MMA this warp issued finish before TMEM is released.
    if (leader) mma_commit(bar(Cfg::kBarDrain + tile));
    __syncwarp();
    drain_wait(bar(Cfg::kBarDrain + tile), 0);
  }
}

// One step of a softmax warp: the scores of its 16-row slice of a query tile for one key
// block -> P in TMEM (fp16), running max / sum updated, O rescaled in TMEM when the max was
// raised. Fragments are TMEM 16x256b: lane 4g + q holds rows g and g + 8 of the slice and,
// of every group of 8 key columns, columns 2q and 2q + 1; the four threads of a row are
// neighbouring lanes of one warp, so a row reduction is two shuffles and no two warps ever
// wait for each other. Returns false if the CTA is unwinding.
template <class Cfg>
__device__ __forceinline__ bool softmax_step(const FwdParams& p, uint32_t bars, uint32_t tS,
                                             uint32_t tP, uint32_t tO, int tile, int lane, int g,
                                             int j, int row0, bool first, float (&m_run)[2],
                                             float (&l_run)[2], const Watchdog& wd) {
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  auto f = [](uint32_t u) { return __uint_as_float(u); };
  const float c = p.scale_log2;
  if (!wait_warp(bar(Cfg::kBarSFull + tile), static_cast<uint32_t>(g) & 1u, wd, kSiteSoftSFull))
    return false;
  tc_fence_after();
  uint32_t sr[64];  // sr[4i + e]: row g + 8 (e / 2), key 8i + 2q + e % 2
  tmem_ld_16x256b_sync(tS, sr);
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(bar(Cfg::kBarSFree + tile));

  if (j == p.sc.nkb - 1) {
    // last key block of the sequence: keys past N score -inf
    const int valid = p.n - j * Cfg::kKeys;
    if (valid < Cfg::kKeys) {
      const int q2 = 2 * (lane & 3);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (8 * i + q2 + (e & 1) >= valid) sr[4 * i + e] = __float_as_uint(-INFINITY);
      }
    }
  }
  if constexpr (Cfg::kCausal) {
    // Keys after the query row score -inf. row0 is the first query row of this warp's 16-row
    // slice; only blocks that reach past it need the per-element test.
    const int key0 = j * Cfg::kKeys;
    if (key0 + Cfg::kKeys - 1 > row0) {
      const int t0 = row0 + (lane >> 2) - key0;  // row g: column c is masked when c > t0
      const int q2 = 2 * (lane & 3);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (8 * i + q2 + (e & 1) > t0 + 8 * (e >> 1)) sr[4 * i + e] = __float_as_uint(-INFINITY);
      }
    }
  }

  // This thread's row maxima: two 3-input max chains per row over its 32 scores.
  float mloc[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float a = fmaxf(f(sr[2 * r]), f(sr[2 * r + 1]));
    float b = fmaxf(f(sr[4 + 2 * r]), f(sr[5 + 2 * r]));
#pragma unroll
    for (int i = 2; i < 16; i += 2) {
      a = max3(a, f(sr[4 * i + 2 * r]), f(sr[4 * i + 2 * r + 1]));
      b = max3(b, f(sr[4 * i + 4 + 2 * r]), f(sr[4 * i + 5 + 2 * r]));
    }
    mloc[r] = fmaxf(a, b);
  }
  // The reference max is raised only when some row of the warp grew past the threshold. A
  // row grows iff one of its four threads holds a score past it (c > 0: scaling preserves
  // the order), so the vote runs on the thread maxima and the row maxima are combined by
  // shuffles only on that rare path; otherwise the reference max stays and alpha = 1.
  const bool grow = __any_sync(0xffffffffu, mloc[0] * c > m_run[0] + Cfg::kRescaleThreshold ||
                                                mloc[1] * c > m_run[1] + Cfg::kRescaleThreshold);
  float alpha[2] = {1.0f, 1.0f};
  if (grow) {
#pragma unroll
    for (int r = 0; r < 2; ++r) mloc[r] = fmaxf(mloc[r], __shfl_xor_sync(0xffffffffu, mloc[r], 1));
#pragma unroll
    for (int r = 0; r < 2; ++r) mloc[r] = fmaxf(mloc[r], __shfl_xor_sync(0xffffffffu, mloc[r], 2));
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float m_use = fmaxf(m_run[r], mloc[r] * c);
      // 0 on a unit's first block (m_run = -inf); 1 while every key so far is masked
      // (causal, m_use = -inf), without an -inf - -inf
      if (!(Cfg::kCausal && m_use == -INFINITY)) alpha[r] = ex2_approx(m_run[r] - m_use);
      m_run[r] = m_use;
    }
  }
  uint64_t negm2[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    // every key so far masked for this row (causal, possible in a piece of a query block):
    // O and the row sum are still zero, and p = 2^(-inf - 0) = 0
    negm2[r] = f2_splat(Cfg::kCausal && m_run[r] == -INFINITY ? 0.0f : -m_run[r]);
  }

  // Scale-subtract and row sums run on packed pairs (fma/add .f32x2); pair k is row k % 2.
  // Pairs whose index has its bit set in kPolyMask take exp2 from the FMA-pipe polynomial,
  // the others from MUFU.
  const uint64_t c2 = f2_splat(c);
  uint32_t pk[32];  // pk[2i + e]: row g + 8e, keys 8i + 2q, 8i + 2q + 1 (16x128b fragment)
  uint64_t acc[4];  // four partial row-sum chains, started by the first four pairs
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const uint64_t x = f2_fma(f2_pack(f(sr[2 * k]), f(sr[2 * k + 1])), c2, negm2[k & 1]);
    float x0, x1, e0, e1;
    f2_unpack(x, x0, x1);
    if ((Cfg::kPolyMask >> (k & 7)) & 1u) {
      exp2_poly_pair(x0, x1, e0, e1);
    } else {
      e0 = ex2_approx(x0);
      e1 = ex2_approx(x1);
    }
    acc[k & 3] = k < 4 ? f2_pack(e0, e1) : f2_add(acc[k & 3], f2_pack(e0, e1));
    pk[k] = pack_pair<Cfg::kBF16>(e0, e1);
  }
  float s0, s1, t0, t1;
  f2_unpack(f2_add(acc[0], acc[2]), s0, s1);
  f2_unpack(f2_add(acc[1], acc[3]), t0, t1);
  l_run[0] = l_run[0] * alpha[0] + (s0 + s1);
  l_run[1] = l_run[1] * alpha[1] + (t0 + t1);

  // P and O are free once the previous O += P V has completed.
  if (g > 0) {
    if (!wait_warp(bar(Cfg::kBarODone + tile), static_cast<uint32_t>(g - 1) & 1u, wd,
                   kSiteSoftODone))
      return false;
    tc_fence_after();
  }
  tmem_st_16x128b_x16(tP, pk);
  if (grow && !first) {
    uint32_t o[Cfg::kHeadDim / 2];  // o[4i + e]: row g + 8 (e / 2), d 8i + 2q + e % 2
    tmem_ld_16x256b_sync(tO, o);
#pragma unroll
    for (int k = 0; k < Cfg::kHeadDim / 2; ++k)
      o[k] = __float_as_uint(f(o[k]) * alpha[(k >> 1) & 1]);
    tmem_st_16x256b(tO, o);
  }
  tmem_wait_st();
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(bar(Cfg::kBarPFull + tile));
  return true;
}

// Query tile of softmax warp w. With two tiles the tiles alternate every four warps
// (0-3, 8-11: tile 0; 4-7, 12-15: tile 1): a sub-partition's four softmax warps are w, w + 4,
// w + 8 and w + 12 in issue priority, so each tile gets one of the first two and one of the
// last two (with tiles by blocks of eight, tile 0 held both favoured warps of every
// sub-partition and tile 1 waited on its two others; this measured 0.3-0.7% fewer cycles).
template <class Cfg>
__device__ __forceinline__ int softmax_tile(int warp) {
  return Cfg::NQ == 2 ? (warp >> 2) & 1 : 0;
}

template <class Cfg>
__device__ __forceinline__ void softmax_role(const FwdParams& p, uint8_t* smem, uint32_t bars,
                                             uint32_t tmem, int tile, const Watchdog& wd) {
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Warp w of the tile may only reach TMEM lane quadrant w % 4; the two warps of a quadrant
  // take its upper and lower 16 rows.
  // first tile row of this warp: quadrant w % 4, upper or lower half (see softmax_tile)
  const int slice = (warp & 3) * 32 + ((warp >> (Cfg::NQ == 2 ? 3 : 2)) & 1) * 16;
  const int gq = lane >> 2;                                     // rows slice + gq, + gq + 8
  const int q = lane & 3;
  const uint32_t lane_bits = static_cast<uint32_t>(slice) << 16;
  const uint32_t tS = tmem + lane_bits + Cfg::kColS + 128 * tile;
  const uint32_t tP = tmem + lane_bits + Cfg::kColP + 64 * tile;
  const uint32_t tO = tmem + lane_bits + Cfg::kColO + Cfg::kHeadDim * tile;
  const bool tile_leader = warp == 4 * (Cfg::NQ - 1) * tile && lane == 0;  // first warp of the tile

  int g = 0;  // global step index (phase of the per-step barriers)
  [[maybe_unused]] int stores = 0;  // whole units stored (staging phase; no store warp)
  StepCursor<Cfg::kCausal> cur;
  cur.init(p);
  while (cur.valid()) {
    float m_run[2] = {-INFINITY, -INFINITY};  // running max of s*scale*log2(e), per row
    float l_run[2] = {0.0f, 0.0f};            // this thread's partial row sums
    const int row0 =  // first query row of this warp's slice (causal masking only)
        Cfg::kCausal ? p.q0 + p.sc.qb_of(cur.u) * Cfg::kRowsPerUnit + tile * Cfg::kRows + slice
                     : 0;
    for (int j = cur.j0; j < cur.j1; ++j, ++g) {
      if (!softmax_step<Cfg>(p, bars, tS, tP, tO, tile, lane, g, j, row0, j == cur.j0, m_run,
                             l_run, wd))
        return;
    }
    // ---- unit epilogue (g - 1 is the unit's last step)
    if (!wait_warp(bar(Cfg::kBarODone + tile), static_cast<uint32_t>(g - 1) & 1u, wd,
                   kSiteSoftOFinal))
      return;
    tc_fence_after();
    float l_row[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      l_row[r] = l_run[r] + __shfl_xor_sync(0xffffffffu, l_run[r], 1);
      l_row[r] += __shfl_xor_sync(0xffffffffu, l_row[r], 2);
    }
    uint32_t o[Cfg::kHeadDim / 2];  // o[4i + e]: row gq + 8 (e / 2), d 8i + 2q + e % 2
    tmem_ld_16x256b_sync(tO, o);
    tc_fence_before();
    const int b = cur.seg_idx & 1;
    if (cur.whole(p.sc)) {
      if (Cfg::kLSE && q == 0) {
        // log-sum-exp = ln 2 * (m + log2 l), m in scaled log2 units
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int qrow = p.sc.qb_of(cur.u) * Cfg::kRowsPerUnit + tile * Cfg::kRows +
                           slice + gq + 8 * r;
          if (qrow < p.nq)
            p.lse[static_cast<size_t>(p.sc.head_of(cur.u)) * p.n + qrow] =
                (m_run[r] + log2f(l_row[r])) * 0.6931471805599453f;
        }
      }
      // O / l -> fp16 -> swizzled staging (this tile's slot of the unit's Q buffer) -> TMA.
      uint8_t* stage = smem + Cfg::kQOff + (b * Cfg::NQ + tile) * Cfg::kTileBytes;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = slice + gq + 8 * r;
        const float inv_l = 1.0f / l_row[r];
        // the TMA box layout: box x holds columns [64x, 64x + 64); in a row of kRowBytes
        // the 16-byte chunk c sits at c ^ (row-address bits 7.., the swizzle pattern)
        const int swz = ((row * Cfg::kRowBytes) >> 7) & (Cfg::kSwizzleChunks - 1);
#pragma unroll
        for (int i = 0; i < Cfg::kHeadDim / 8; ++i) {  // 16-byte chunk i, 4 bytes per thread
          const uint32_t w = pack_pair<Cfg::kBF16>(__uint_as_float(o[4 * i + 2 * r]) * inv_l,
                                                   __uint_as_float(o[4 * i + 2 * r + 1]) * inv_l);
          const int x = i / Cfg::kSwizzleChunks, c = i % Cfg::kSwizzleChunks;
          const uint32_t dst = smem_addr(stage + x * Cfg::kBoxBytes + row * Cfg::kRowBytes +
                                         ((c ^ swz) << 4) + 4 * q);
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(dst), "r"(w) : "memory");
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(Cfg::kBarStage + tile));
      if constexpr (!Cfg::kStoreRole) {
        // no store warp: the tile's first warp stores once all eight have written their
        // staging rows, then frees the Q buffer when the store has read it
        if (tile_leader) {
          if (!wait_single(bar(Cfg::kBarStage + tile), static_cast<uint32_t>(stores) & 1u, wd,
                           kSiteSoftStage))
            return;
          const int r0 = p.sc.qb_of(cur.u) * Cfg::kRowsPerUnit + tile * Cfg::kRows;
          if (r0 < p.nq) {
            const HeadBatch ob = head_batch(p, cur.u);
#pragma unroll
            for (int x = 0; x < Cfg::kBoxes; ++x)
              tma_store_4d(&p.tm_o, smem_addr(stage + x * Cfg::kBoxBytes), x * Cfg::kBoxCols,
                           r0, ob.h, ob.b);
            tma_store_commit();
            tma_store_wait_read();
          }
          mbar_arrive(bar(Cfg::kBarQEmpty + b));
        }
        ++stores;
      }
    } else {
      // A piece of a query block: unnormalised O, the row max and the row sum go to this
      // CTA's workspace slot (first or last segment of its range) for the merge kernel.
      float* ws = p.workspace +
                  static_cast<size_t>(2 * blockIdx.x + (cur.first_of_range() ? 0 : 1)) *
                      Cfg::kSlotFloats;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = tile * Cfg::kRows + slice + gq + 8 * r;
        float2* dst = reinterpret_cast<float2*>(ws + static_cast<size_t>(row) * Cfg::kHeadDim);
#pragma unroll
        for (int i = 0; i < Cfg::kHeadDim / 8; ++i)
          dst[4 * i + q] = make_float2(__uint_as_float(o[4 * i + 2 * r]),
                                       __uint_as_float(o[4 * i + 2 * r + 1]));
        if (q == 0) {
          ws[Cfg::kRowsPerUnit * Cfg::kHeadDim + row] = m_run[r];
          ws[Cfg::kRowsPerUnit * (Cfg::kHeadDim + 1) + row] = l_row[r];
        }
      }
      // the Q buffer was only read by this unit's S MMAs, all complete by now
      if (tile_leader) mbar_arrive(bar(Cfg::kBarQEmpty + b));
    }
    cur.next_segment(p);
  }
}

// One thread of the store warp: once the eight softmax warps of a tile have written its
// normalised output into the staging buffer (the unit's Q buffer), store it with TMA, and
// free the Q buffer for the load warp when the stores have read it. Keeping the store's
// issue and read wait here leaves the softmax warps free to start the next unit.
template <class Cfg>
__device__ __forceinline__ void store_role(const FwdParams& p, uint8_t* smem, uint32_t bars,
                                           const Watchdog& wd) {
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  StepCursor<Cfg::kCausal> cur;
  cur.init(p);
  int stores = 0;  // whole units stored so far (phase of the staging barriers)
  while (cur.valid()) {
    if (cur.whole(p.sc)) {
      const int b = cur.seg_idx & 1;
      const HeadBatch ob = head_batch(p, cur.u);
      bool ok = true;
#pragma unroll
      for (int tile = 0; tile < Cfg::NQ; ++tile) {
        if (!wait_single(bar(Cfg::kBarStage + tile), static_cast<uint32_t>(stores) & 1u, wd,
                         kSiteSoftStage)) {
          ok = false;
          break;
        }
        const int r0 = p.sc.qb_of(cur.u) * Cfg::kRowsPerUnit + tile * Cfg::kRows;
        if (r0 < p.nq) {
          const uint32_t stage =
              smem_addr(smem + Cfg::kQOff + (b * Cfg::NQ + tile) * Cfg::kTileBytes);
#pragma unroll
          for (int x = 0; x < Cfg::kBoxes; ++x)
            tma_store_4d(&p.tm_o, stage + x * Cfg::kBoxBytes, x * Cfg::kBoxCols, r0, ob.h, ob.b);
        }
      }
      tma_store_commit();
      if (!ok) break;
      tma_store_wait_read();
#pragma unroll
      for (int tile = 0; tile < Cfg::NQ; ++tile) mbar_arrive(bar(Cfg::kBarQEmpty + b));
      ++stores;
    }
    cur.next_segment(p);
  }
  // Unwinding or done: shared memory must outlive every store's read of it.
  tma_store_wait_read();
}

template <int NQ, int STAGES, bool CAUSAL, bool BF16, int D, bool LSE>
__global__ void __launch_bounds__(FwdConfig<NQ, STAGES, CAUSAL, BF16, D, LSE>::kThreads, 1)
    mfa_fwd_kernel(const __grid_constant__ FwdParams p) {
  using Cfg = FwdConfig<NQ, STAGES, CAUSAL, BF16, D, LSE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const uint32_t bars = smem_addr(smem + Cfg::kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kTmemSlotOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kAbortOff);

  // The split-mode merge kernel may be scheduled now; it waits for this grid to complete
  // before reading anything this grid writes.
  if (threadIdx.x == 0) grid_dependents_launch();
  // This grid is itself launched as a programmatic dependent of the stream's previous kernel:
  // the set-up below (barriers, TMEM) may overlap that kernel's tail; every warp then waits
  // for that kernel's completion before its role starts, i.e. before any global memory
  // access and before any bounded wait (whose limit would otherwise run during that kernel).
  // The load thread initialises the barriers and goes straight on to its first copies; the
  // other warps wait on named barrier 1 for the barriers and for warp 0's TMEM allocation
  // (the load warp only arrives there), so the first Q/K/V loads leave while TMEM is set up.
  uint32_t tmem = 0;  // TMEM base (all warps but the load warp)
  if (warp == Cfg::kLoadWarp) {
    if (lane == 0) {
      *abort_flag = 0;
      for (int b = 0; b < 2; ++b) {
        mbar_init(bars + 8 * (Cfg::kBarQFull + b), 1);
        mbar_init(bars + 8 * (Cfg::kBarQEmpty + b), Cfg::NQ);  // one arrive per tile epilogue
      }
      for (int s = 0; s < STAGES; ++s) {
        mbar_init(bars + 8 * (Cfg::kBarKFull + s), 1);
        mbar_init(bars + 8 * (Cfg::kBarKEmpty + s), Cfg::NQ);
        mbar_init(bars + 8 * (Cfg::kBarVFull + s), 1);
        mbar_init(bars + 8 * (Cfg::kBarVEmpty + s), Cfg::NQ);
      }
      for (int i = 0; i < NQ; ++i) {
        mbar_init(bars + 8 * (Cfg::kBarSFull + i), 1);
        mbar_init(bars + 8 * (Cfg::kBarSFree + i), 8);  // one arrive per softmax warp of tile i
        mbar_init(bars + 8 * (Cfg::kBarPFull + i), 8);
        mbar_init(bars + 8 * (Cfg::kBarODone + i), 1);
      }
      for (int i = 0; i < NQ; ++i) mbar_init(bars + 8 * (Cfg::kBarStage + i), 8);
      for (int i = 0; i < NQ; ++i) mbar_init(bars + 8 * (Cfg::kBarDrain + i), 1);
      mbar_init_fence();
    }
    __syncwarp();
    named_bar_arrive(1, Cfg::kThreads);
    if constexpr (Cfg::kRebalanceRegs) setmaxnreg_dec<Cfg::kControlRegs>();
    const Watchdog wd{abort_flag, p.status, p.timeout_ns};
    grid_dependency_wait();
    if (lane == 0) load_role<Cfg>(p, smem, bars, wd);
  } else {
    if (warp == 0) {
      tmem_alloc(smem_addr(tmem_slot), Cfg::kTmemCols);
      tmem_relinquish();
    }
    tc_fence_before();
    named_bar_sync(1, Cfg::kThreads);
    tc_fence_after();
    tmem = *tmem_slot;
    grid_dependency_wait();
    const Watchdog wd{abort_flag, p.status, p.timeout_ns};
    if (warp < Cfg::kSoftmaxWarps) {
      if constexpr (Cfg::kRebalanceRegs) setmaxnreg_inc<Cfg::kSoftmaxRegs>();
      softmax_role<Cfg>(p, smem, bars, tmem, softmax_tile<Cfg>(warp), wd);
    } else {
      if constexpr (Cfg::kRebalanceRegs) setmaxnreg_dec<Cfg::kControlRegs>();
      if (warp == Cfg::kMmaWarp || (Cfg::NQ == 2 && warp == Cfg::kMmaWarp2)) {
        mma_role<Cfg>(p, smem, bars, tmem, wd, warp == Cfg::kMmaWarp ? 0 : 1);
      } else if (Cfg::kStoreRole && warp == Cfg::kStoreWarp) {
        if (lane == 0) store_role<Cfg>(p, smem, bars, wd);
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
}

// ---------------------------------------------------------------- split-mode merge
struct MergeParams {
  void* out;          // fp16 / bf16, row (b, h, n) at b * stride_b + h * stride_h + n * stride_n
  float* lse;         // optional [BH][N] natural-log log-sum-exp (null: not written)
  const float* workspace;
  int n;              // rows per head of lse
  int nq;             // query rows per head in this launch (out starts at the first)
  int heads;
  long long stride_b, stride_h, stride_n;  // in elements
  Schedule sc;
  int ctas;           // grid size of the forward kernel whose pieces are merged
};

// One CTA per forward CTA c; it merges the query block that starts inside c's range and
// continues past it (if any): every piece's O is rescaled to the common row max, summed,
// divided by the rescaled sum of row sums, rounded to fp16 / bf16. Four threads per query
// row, each on every fourth 16-byte chunk of it, so a warp reads 8 rows x 256 contiguous bytes.
// Launched as a programmatic dependent of the forward kernel: all index work (which query
// block, how many pieces, where the row goes) runs before griddepcontrol.wait and overlaps
// the forward kernel's tail; after the wait the pieces are read two at a time for D <= 64
// (one L2 round trip per pair; one at a time for D = 128, within the register budget) and
// folded into a running max, sum and O.
constexpr int kMergeThreadsPerRow = 4;

template <int kRowsPerUnit, int kSlotFloats, bool kCausal, bool kBF16, int kD, bool kLSE>
__global__ void __launch_bounds__(kRowsPerUnit * kMergeThreadsPerRow)
    mfa_merge_kernel(const MergeParams mp) {
  constexpr int kChunks = kD / 4 / kMergeThreadsPerRow;  // float4 chunks per thread
  constexpr int kOffM = kRowsPerUnit * kD;               // row maxima within a slot
  constexpr int kOffL = kRowsPerUnit * (kD + 1);         // row sums within a slot
  constexpr int kBatch = kChunks <= 4 ? 2 : 1;           // pieces read per round trip
  const int c = static_cast<int>(blockIdx.x);
  long long b0, b1;
  mp.sc.range(c, b0, b1);
  int u = 0, j = 0;
  if (b1 > b0) mp.sc.locate<kCausal>(b1 - 1, u, j);  // query block holding c's last step
  const long long u0 = mp.sc.unit_first<kCausal>(u);
  const long long u1 = u0 + mp.sc.steps_of<kCausal>(mp.sc.qb_of(u));
  // Merged here only if it starts inside c and ends past it.
  if (!(b1 > b0 && u1 > b1 && u0 >= b0)) {
    grid_dependency_wait();
    return;
  }
  // Pieces: c's last segment (its first too if c's range starts exactly at u), then the
  // first segment of every following CTA whose range starts before the query block ends.
  int pieces = 1;
  for (int cc = c + 1; cc < mp.ctas; ++cc) {
    long long s0, s1;
    mp.sc.range(cc, s0, s1);
    if (s0 >= u1) break;
    ++pieces;
  }
  const int r = static_cast<int>(threadIdx.x) / kMergeThreadsPerRow;
  const int k = static_cast<int>(threadIdx.x) % kMergeThreadsPerRow;
  const int bh = mp.sc.head_of(u);
  const int qrow = (u - bh * mp.sc.q_blocks) * kRowsPerUnit + r;
  const long long offset = static_cast<long long>(bh / mp.heads) * mp.stride_b +
                           static_cast<long long>(bh % mp.heads) * mp.stride_h +
                           static_cast<long long>(qrow) * mp.stride_n;
  // Slot of piece i: CTA c's second slot unless its range starts at u; slot 0 of the others.
  const float* first = mp.workspace + static_cast<size_t>(2 * c + (b0 == u0 ? 0 : 1)) * kSlotFloats;
  auto piece = [&](int i) {
    return i == 0 ? first : mp.workspace + static_cast<size_t>(2 * (c + i)) * kSlotFloats;
  };
  grid_dependency_wait();
  if (qrow >= mp.nq) return;

  // Piece 0 holds key block 0, so its row max is finite for every row (causal included) and
  // the running max is finite from the first pair on; a fully masked later piece has
  // m = -inf and weight 0.
  float m_run = -INFINITY, l = 0.0f;
  float4 acc[kChunks];
#pragma unroll
  for (int i = 0; i < kChunks; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = 0; i < pieces; i += kBatch) {
    float m[kBatch], ls[kBatch];
    float4 o[kBatch][kChunks];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      // a missing last piece of the batch re-reads piece i with m = -inf, i.e. weight 0
      const bool here = i + b < pieces;
      const float* ws = piece(here ? i + b : i);
      m[b] = here ? ws[kOffM + r] : -INFINITY;
      ls[b] = ws[kOffL + r];
      const float4* src = reinterpret_cast<const float4*>(ws + static_cast<size_t>(r) * kD);
#pragma unroll
      for (int q = 0; q < kChunks; ++q) o[b][q] = src[kMergeThreadsPerRow * q + k];
    }
    float m_new = m_run;
#pragma unroll
    for (int b = 0; b < kBatch; ++b) m_new = fmaxf(m_new, m[b]);
    const float s = ex2_approx(m_run - m_new);  // 0 on the first batch (m_run = -inf)
    l *= s;
#pragma unroll
    for (int q = 0; q < kChunks; ++q) {
      acc[q].x *= s;
      acc[q].y *= s;
      acc[q].z *= s;
      acc[q].w *= s;
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const float w = ex2_approx(m[b] - m_new);
      l += w * ls[b];
#pragma unroll
      for (int q = 0; q < kChunks; ++q) {
        acc[q].x += w * o[b][q].x;
        acc[q].y += w * o[b][q].y;
        acc[q].z += w * o[b][q].z;
        acc[q].w += w * o[b][q].w;
      }
    }
    m_run = m_new;
  }
  if (kLSE && k == 0)
    mp.lse[static_cast<size_t>(bh) * mp.n + qrow] = (m_run + log2f(l)) * 0.6931471805599453f;
  const float inv_l = 1.0f / l;
  uint2* dst = reinterpret_cast<uint2*>(static_cast<uint16_t*>(mp.out) + offset);
#pragma unroll
  for (int q = 0; q < kChunks; ++q) {
    uint2 w;
    w.x = pack_pair<kBF16>(acc[q].x * inv_l, acc[q].y * inv_l);
    w.y = pack_pair<kBF16>(acc[q].z * inv_l, acc[q].w * inv_l);
    dst[kMergeThreadsPerRow * q + k] = w;
  }
}

}  // namespace mfa
