// FlashAttention backward for sm_100a (D = 64, fp16 or bf16, optional causal mask): the last
// "next" item of the reference's README (backward pass, README.md:125). Not a translation: the
// reference has no backward.
//
// Given q, k, v, o, dO and the forward's row log-sum-exp L (natural log), with
// P = exp(scale * q k^T - L) and D_i = rowsum(dO ⊙ o):
//   dV = P^T dO,   dS = P ⊙ (dO v^T - D),   dQ = scale * dS k,   dK = scale * dS^T q.
// Two passes of one persistent kernel, no atomics (dQ gets its own pass, which recomputes S
// and dP, instead of accumulating across CTAs):
//   dQ pass  : a CTA keeps a 128-row block of q and dO resident and streams the k, v blocks;
//              S = q k^T and dP = dO v^T (tcgen05 SS MMAs into TMEM), dS in registers (fp16
//              or bf16 into TMEM), dQ += dS k (TS MMA; k read MN-major, no transpose).
//   dK/dV pass: a CTA keeps a 128-row block of k and v resident and streams the q, dO blocks
//              with their L and D slices; S^T = k q^T and dP^T = v dO^T, P^T and dS^T in TMEM,
//              dV += P^T dO and dK += dS^T q.
// TMEM (columns): S or S^T [0,128), dP or dP^T [128,256), P^T / dS [256,320), dS^T [320,384),
// accumulators dQ [320,384) or dV [384,448) and dK [448,512).
// Warp roles as in the forward kernel (csrc/mfa_fwd_kernel.cuh): 16 softmax-side warps on
// 16x256b TMEM fragments (lane 4g + q: rows g and g + 8 of a 16-row slice, columns 2q, 2q + 1
// of every 8), one MMA warp (one elected lane issues), one TMA warp; every wait is bounded.
// The backward needs no row reductions (L and D come precomputed), so the 128 columns of a
// block are split between two warps per 16-row slice: warp w takes TMEM lane quadrant w % 4,
// slice half (w / 4) % 2 and column half w / 8, which doubles the warps that hide each other's
// latencies at the same TMEM footprint.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "mfa_common.cuh"
#include "mfa_exp2.cuh"
#include "mfa_ptx.cuh"

namespace mfa {

struct BwdParams {
  // {64, N, H, B} tensor maps, box {64, 128, 1, 1}, 128-byte swizzle (as the forward's)
  CUtensorMap tm_x, tm_y;    // resident: dQ pass q, dO; dK/dV pass k, v
  CUtensorMap tm_s0, tm_s1;  // streamed: dQ pass k, v; dK/dV pass q, dO
  CUtensorMap tm_o0, tm_o1;  // outputs: dQ pass dQ; dK/dV pass dK (o0), dV (o1)
  int n;                     // sequence length
  int heads;
  int bh;                    // batch * heads
  int blocks;                // 128-row blocks per head: ceil(N / 128)
  float scale;               // softmax scale (multiplies q.k; dQ and dK are scaled by it)
  float scale_log2;          // scale * log2(e)
  const float* lse2;         // [bh][blocks * 128]: L * log2(e), +inf past N
  const float* di;           // [bh][blocks * 128]: rowsum(dO ⊙ o), 0 past N
  unsigned long long timeout_ns;
  int* status;
  // CTAs [cta0, cta0 + ctas) of the launch run this pass
  int cta0;
  int ctas;
  int by_length;  // causal only: deal units out by length (below), else strided
  int reverse;    // CTA cta0 + c deals as CTA ctas - 1 - c (the second pass of a mixed launch)
};

template <bool kDKV_, bool kCausal_, bool kBF16_>
struct BwdConfig {
  static constexpr bool kDKV = kDKV_;  // dK/dV pass (k, v resident) or dQ pass (q, dO resident)
  static constexpr bool kCausal = kCausal_;
  static constexpr bool kBF16 = kBF16_;
  static constexpr int kHeadDim = 64;
  static constexpr int kRows = 128;  // resident rows per unit (M of every MMA)
  static constexpr int kCols = 128;  // streamed rows per step
  static constexpr int kTileBytes = kRows * kHeadDim * 2;
  static constexpr int STAGES = 3;
  static constexpr int kSoftmaxWarps = 16;  // 16 rows x 64 columns each
  // Two MMA issuers: warp 16 the S and dP products (SS), warp 19 the accumulations (TS). One
  // thread issues a tcgen05.mma only every few tens of cycles, and a step has 24 products in
  // the dK/dV pass (16 in the dQ pass), most of them 128x64x16 (32 tensor-core cycles each).
  static constexpr int kMmaWarp = 16;
  static constexpr int kLoadWarp = 17;
  static constexpr int kStoreWarp = 18;  // TMA stores of finished units' gradients
  static constexpr int kAccWarp = 19;
  // As in the forward kernel: 640 threads (the two MMA warps, the load and the store warp fill
  // a fifth warpgroup) launch with 96 registers; setmaxnreg moves the control warpgroup to 64 and
  // the four softmax-side warpgroups to 104 (512 x 104 + 128 x 64 = 640 x 96; per SM
  // sub-partition 4 x 104 + 64 <= 512 registers per lane).
  static constexpr int kThreads = 32 * 20;
  static constexpr int kSoftmaxRegs = 104;
  static constexpr int kControlRegs = 64;

  // shared memory (1024-aligned base)
  static constexpr int kResOff = 0;                                  // [2 buffers][x, y]
  static constexpr int kStrOff = kResOff + 2 * 2 * kTileBytes;       // [STAGES][tile 0, tile 1]
  static constexpr int kVecBytes = 2 * kCols * 4;                    // L2 slice, D slice
  static constexpr int kVecOff = kStrOff + STAGES * 2 * kTileBytes;  // [STAGES] (dK/dV pass)
  static constexpr int kBarOff = kVecOff + (kDKV ? STAGES * kVecBytes : 0);
  static constexpr int kBarResFull = 0;   // [2]
  static constexpr int kBarResEmpty = 2;  // [2]
  static constexpr int kBarStrFull = 4;   // [STAGES]
  static constexpr int kBarStrEmpty = kBarStrFull + STAGES;
  static constexpr int kBarSSFull = kBarStrEmpty + STAGES;  // S and dP computed
  static constexpr int kBarSSFree = kBarSSFull + 1;         // S and dP read by all 16 warps
  static constexpr int kBarOpFull = kBarSSFree + 1;         // fp16 operands written (16 warps)
  static constexpr int kBarAccDone = kBarOpFull + 1;        // TS MMAs of a step completed
  static constexpr int kBarStage = kBarAccDone + 1;         // output staging written (16 warps)
  static constexpr int kBarDrain = kBarStage + 1;  // [2]: one per MMA issuer
  static constexpr int kNumBars = kBarDrain + 2;
  static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr int kAbortOff = kTmemSlotOff + 4;
  static constexpr int kSmemBytes = kAbortOff + 4 + 1024;

  static constexpr int kTmemCols = 512;
  static constexpr int kColS = 0;
  static constexpr int kColDP = 128;
  static constexpr int kColOp0 = 256;  // dQ pass: dS; dK/dV pass: P^T
  static constexpr int kColOp1 = 320;  // dK/dV pass: dS^T
  static constexpr int kColAcc0 = kDKV ? 384 : 320;  // dQ pass: dQ; dK/dV pass: dV
  static constexpr int kColAcc1 = 448;               // dK/dV pass: dK
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// Units are (batch * head, 128-row block) pairs, u = bh * blocks + block.
// dQ pass: unit = query block b, steps = key blocks [0, b + 1) with the causal mask, else all.
// dK/dV pass: unit = key block b, steps = query blocks [b, blocks) with the mask, else all.
// By default the pass's CTA c takes units c, c + ctas, ... (neighbouring CTAs on neighbouring
// blocks of a head, so the streamed blocks come from L2). With the mask and few units per CTA
// (by_length) unit lengths, which run from 1 to `blocks`, would leave CTAs unevenly loaded:
// the units are then taken in order of decreasing length (i = 0, 1, ...: block b = blocks - 1
// - i / bh for dQ, i / bh for dK/dV, head i % bh) and dealt out boustrophedon (wave k goes to
// CTAs 0..ctas-1 for even k, back from ctas-1 for odd k), which evens out the step counts.
template <class Cfg>
struct BwdCursor {
  int u;       // unit
  int j;       // streamed block of the current step
  int j0, j1;  // streamed blocks [j0, j1) of u
  int seg;     // units started by this CTA so far - 1

  __device__ void bounds(const BwdParams& p) {
    const int blk = u % p.blocks;
    if (Cfg::kDKV) {
      j0 = Cfg::kCausal ? blk : 0;
      j1 = p.blocks;
    } else {
      j0 = 0;
      j1 = Cfg::kCausal ? blk + 1 : p.blocks;
    }
    j = j0;
  }
  // Unit of this CTA's k-th assignment, or -1 past the end.
  __device__ static int unit_at(const BwdParams& p, int k) {
    // units <= 2^31 - 2^16 (checked by the launcher), k * ctas <= units: 32-bit arithmetic
    const int c0 = static_cast<int>(blockIdx.x) - p.cta0;
    const int c = p.reverse ? p.ctas - 1 - c0 : c0;
    const int units = p.bh * p.blocks;
    if (!Cfg::kCausal || !p.by_length) {
      const int u = k * p.ctas + c;
      return u < units ? u : -1;
    }
    const int i = k * p.ctas + ((k & 1) ? p.ctas - 1 - c : c);
    if (i >= units) return -1;
    const int wave = i / p.bh, head = i - wave * p.bh;
    const int blk = Cfg::kDKV ? wave : p.blocks - 1 - wave;
    return head * p.blocks + blk;
  }
  __device__ void init(const BwdParams& p) {
    seg = 0;
    u = unit_at(p, 0);
    if (u >= 0) {
      bounds(p);
    } else {
      u = 0;
      j = j0 = j1 = 0;
    }
  }
  __device__ bool valid() const { return j < j1; }
  __device__ bool first_step() const { return j == j0; }
  __device__ void step(const BwdParams& p) {
    if (++j >= j1) {
      const int next = unit_at(p, seg + 1);
      if (next >= 0) {
        u = next;
        bounds(p);
        ++seg;
      }
    }
  }
};

__device__ __forceinline__ HeadBatch bwd_head_batch(const BwdParams& p, int u) {
  const int bh = u / p.blocks;
  return {bh % p.heads, bh / p.heads};
}

template <class Cfg>
__device__ __forceinline__ void bwd_load_role(const BwdParams& p, uint8_t* smem, uint32_t bars,
                                              const Watchdog& wd) {
  constexpr int ST = Cfg::STAGES;
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  const uint32_t sbase = smem_addr(smem);
  tma_prefetch_desc(&p.tm_x);
  tma_prefetch_desc(&p.tm_y);
  tma_prefetch_desc(&p.tm_s0);
  tma_prefetch_desc(&p.tm_s1);
  const uint64_t keep = l2_policy_evict_last();  // streamed blocks are re-read by other units
  BwdCursor<Cfg> cur;
  cur.init(p);
  int g = 0;
  int res_loaded = 0, str_issued = 0;
  while (cur.valid()) {
    const HeadBatch hb = bwd_head_batch(p, cur.u);
    if (cur.first_step()) {
      const int s = cur.seg, b = s & 1;
      if (!wait_single(bar(Cfg::kBarResEmpty + b), (static_cast<uint32_t>(s >> 1) & 1u) ^ 1u, wd,
                       kSiteLoadQEmpty))
        break;
      mbar_arrive_expect_tx(bar(Cfg::kBarResFull + b), 2 * Cfg::kTileBytes);
      const int row = (cur.u % p.blocks) * Cfg::kRows;
      const uint32_t dst = sbase + Cfg::kResOff + b * 2 * Cfg::kTileBytes;
      tma_load_4d(dst, &p.tm_x, bar(Cfg::kBarResFull + b), 0, row, hb.h, hb.b);
      tma_load_4d(dst + Cfg::kTileBytes, &p.tm_y, bar(Cfg::kBarResFull + b), 0, row, hb.h, hb.b);
      res_loaded = s + 1;
    }
    const int st = g % ST;
    if (!wait_single(bar(Cfg::kBarStrEmpty + st), (static_cast<uint32_t>(g / ST) & 1u) ^ 1u, wd,
                     kSiteLoadKEmpty))
      break;
    mbar_arrive_expect_tx(bar(Cfg::kBarStrFull + st),
                          2 * Cfg::kTileBytes + (Cfg::kDKV ? Cfg::kVecBytes : 0));
    const int row = cur.j * Cfg::kCols;
    const uint32_t dst = sbase + Cfg::kStrOff + st * 2 * Cfg::kTileBytes;
    tma_load_4d_hint(dst, &p.tm_s0, bar(Cfg::kBarStrFull + st), 0, row, hb.h, hb.b, keep);
    tma_load_4d_hint(dst + Cfg::kTileBytes, &p.tm_s1, bar(Cfg::kBarStrFull + st), 0, row, hb.h,
                     hb.b, keep);
    if (Cfg::kDKV) {
      // L2 and D of the 128 streamed queries (padded arrays: 512-byte aligned slices)
      const size_t off = static_cast<size_t>(cur.u / p.blocks) * p.blocks * Cfg::kCols + row;
      const uint32_t vdst = sbase + Cfg::kVecOff + st * Cfg::kVecBytes;
      bulk_load(vdst, p.lse2 + off, Cfg::kCols * 4, bar(Cfg::kBarStrFull + st));
      bulk_load(vdst + Cfg::kCols * 4, p.di + off, Cfg::kCols * 4, bar(Cfg::kBarStrFull + st));
    }
    str_issued = g + 1;
    ++g;
    cur.step(p);
  }
  if (*wd.abort) {
    for (int b = 0; b < 2; ++b) {
      int last = -1;
      for (int s = b; s < res_loaded; s += 2) last = s;
      if (last >= 0) drain_wait(bar(Cfg::kBarResFull + b), static_cast<uint32_t>(last >> 1) & 1u);
    }
    for (int st = 0; st < ST; ++st) {
      int last = -1;
      for (int x = st; x < str_issued; x += ST) last = x;
      if (last >= 0) drain_wait(bar(Cfg::kBarStrFull + st), static_cast<uint32_t>(last / ST) & 1u);
    }
  }
}

// kAcc false: the S and dP products of every step (warp kMmaWarp); kAcc true: the
// accumulations into dQ, or dV and dK (warp kAccWarp). Both read the streamed stage, whose
// empty barrier counts one commit from each.
template <class Cfg, bool kAcc>
__device__ __forceinline__ void bwd_mma_role(const BwdParams& p, uint8_t* smem, uint32_t bars,
                                             uint32_t tmem, const Watchdog& wd) {
  constexpr int ST = Cfg::STAGES;
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  const uint32_t sbase = smem_addr(smem);
  constexpr uint32_t kIdescSS = idesc_f16_f32(128, 128, false, Cfg::kBF16);
  constexpr uint32_t kIdescTS = idesc_f16_f32(128, 64, true, Cfg::kBF16);
  constexpr uint32_t kHi = smem_desc_hi(1024, kSwizzle128B);
  constexpr uint32_t kTile = Cfg::kTileBytes >> 4;
  const uint32_t res_lo = smem_desc_lo(sbase + Cfg::kResOff, 16);
  const uint32_t str_lo = smem_desc_lo(sbase + Cfg::kStrOff, 16);
  const uint32_t str_mn_lo = smem_desc_lo(sbase + Cfg::kStrOff, Cfg::kTileBytes);
  const bool leader = elect_one();
  bool issued_any = false;

  BwdCursor<Cfg> cs, cp;
  cs.init(p);
  cp.init(p);
  int gs = 0, gp = 0;
  // S and dP of step gs once the softmax warps have read those of step gs - 1.
  auto issue_ss = [&]() -> bool {
    const int b = cs.seg & 1;
    if (cs.first_step()) {
      if (!wait_warp(bar(Cfg::kBarResFull + b), static_cast<uint32_t>(cs.seg >> 1) & 1u, wd,
                     kSiteMmaQ))
        return false;
    }
    const int st = gs % ST;
    if (!wait_warp(bar(Cfg::kBarStrFull + st), static_cast<uint32_t>(gs / ST) & 1u, wd, kSiteMmaK))
      return false;
    if (gs > 0) {
      if (!wait_warp(bar(Cfg::kBarSSFree), static_cast<uint32_t>(gs - 1) & 1u, wd, kSiteMmaSFree))
        return false;
    }
    tc_fence_after();
    if (leader) {
      const uint32_t xd = res_lo + b * 2 * kTile, yd = xd + kTile;
      const uint32_t s0 = str_lo + st * 2 * kTile, s1 = s0 + kTile;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)  // S = x s0^T
        mma_ss(tmem + Cfg::kColS, desc_join(xd + 2 * kk, kHi), desc_join(s0 + 2 * kk, kHi),
               kIdescSS, kk > 0 ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)  // dP = y s1^T
        mma_ss(tmem + Cfg::kColDP, desc_join(yd + 2 * kk, kHi), desc_join(s1 + 2 * kk, kHi),
               kIdescSS, kk > 0 ? 1u : 0u);
      mma_commit(bar(Cfg::kBarSSFull));
      mma_commit(bar(Cfg::kBarStrEmpty + st));
    }
    __syncwarp();
    issued_any = true;
    ++gs;
    cs.step(p);
    return true;
  };

  if (!kAcc) {
    while (cs.valid())
      if (!issue_ss()) goto unwind;
  }
  while (kAcc && cp.valid()) {
    {
      const int st = gp % ST;
      // the stage's tiles are this thread's operands too
      if (!wait_warp(bar(Cfg::kBarStrFull + st), static_cast<uint32_t>(gp / ST) & 1u, wd,
                     kSiteMmaK))
        goto unwind;
      if (!wait_warp(bar(Cfg::kBarOpFull), static_cast<uint32_t>(gp) & 1u, wd, kSiteMmaPFull))
        goto unwind;
      tc_fence_after();
      if (leader) {
        const bool fresh = cp.first_step();
        const uint32_t s0 = str_mn_lo + st * 2 * kTile, s1 = s0 + kTile;
        if (Cfg::kDKV) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // dV += P^T dO
            mma_ts(tmem + Cfg::kColAcc0, tmem + Cfg::kColOp0 + 8 * kk,
                   desc_join(s1 + 128 * kk, kHi), kIdescTS, (!fresh || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // dK += dS^T q
            mma_ts(tmem + Cfg::kColAcc1, tmem + Cfg::kColOp1 + 8 * kk,
                   desc_join(s0 + 128 * kk, kHi), kIdescTS, (!fresh || kk > 0) ? 1u : 0u);
        } else {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // dQ += dS k
            mma_ts(tmem + Cfg::kColAcc0, tmem + Cfg::kColOp0 + 8 * kk,
                   desc_join(s0 + 128 * kk, kHi), kIdescTS, (!fresh || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar(Cfg::kBarAccDone));
        mma_commit(bar(Cfg::kBarStrEmpty + st));
      }
      __syncwarp();
      issued_any = true;
      ++gp;
      cp.step(p);
    }
  }
  // Every commit of this pass has arrived before the role returns (the barriers may be
  // initialised again for a second pass).
  if (issued_any) {
    if (leader) mma_commit(bar(Cfg::kBarDrain + (kAcc ? 1 : 0)));
    __syncwarp();
    // on failure the CTA unwinds
    wait_warp(bar(Cfg::kBarDrain + (kAcc ? 1 : 0)), 0, wd, kSiteMmaDrain);
  }
  return;

unwind:
  if (issued_any) {
    if (leader) mma_commit(bar(Cfg::kBarDrain + (kAcc ? 1 : 0)));
    __syncwarp();
    drain_wait(bar(Cfg::kBarDrain + (kAcc ? 1 : 0)), 0);
  }
}

// One step of a softmax-side warp on its 16 rows: P = 2^(S * scale * log2 e - L2), and
// dS = P ⊙ (dP - D). dQ pass: rows are queries, L2 and D are per row; dK/dV pass: rows are
// keys, columns queries, L2 and D come per column from the streamed slices in shared memory.
template <class Cfg>
__device__ __forceinline__ bool bwd_step(const BwdParams& p, uint8_t* smem, uint32_t bars,
                                         uint32_t tS, uint32_t tDP, uint32_t tOp0, uint32_t tOp1,
                                         int lane, int half, int g, int blk, int j, int row0,
                                         const float (&lrow)[2], const float (&drow)[2],
                                         const Watchdog& wd) {
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  auto f = [](uint32_t u) { return __uint_as_float(u); };
  if (!wait_warp(bar(Cfg::kBarSSFull), static_cast<uint32_t>(g) & 1u, wd, kSiteSoftSFull))
    return false;
  tc_fence_after();
  // [4i + e]: row g + 8 (e / 2), column 64 * half + 8i + 2q + e % 2 (tS, tDP already point at
  // this warp's column half)
  uint32_t sr[32], dp[32];
  tmem_ld2_16x256b_sync(tS, sr, tDP, dp);
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(bar(Cfg::kBarSSFree));

  const int q2 = 2 * (lane & 3) + 64 * half;  // first of this thread's columns in a block
  const int gq = lane >> 2;
  if (!Cfg::kDKV) {
    // keys past N (last key block) and, with the mask, keys after the query row
    if (j == p.blocks - 1) {
      const int valid = p.n - j * Cfg::kCols;
      if (valid < Cfg::kCols) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (8 * i + q2 + (e & 1) >= valid) sr[4 * i + e] = __float_as_uint(-INFINITY);
      }
    }
    if (Cfg::kCausal) {
      const int t0 = row0 + gq - j * Cfg::kCols;  // column k masked when k > t0 (+8 for e >= 2)
      if (j * Cfg::kCols + Cfg::kCols - 1 > row0) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (8 * i + q2 + (e & 1) > t0 + 8 * (e >> 1)) sr[4 * i + e] = __float_as_uint(-INFINITY);
      }
    }
  } else if (Cfg::kCausal && j == blk) {
    // diagonal block: queries (columns) before the key row score -inf
    const int t0 = row0 + gq - j * Cfg::kCols;  // column k masked when k < t0 (+8 for e >= 2)
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (8 * i + q2 + (e & 1) < t0 + 8 * (e >> 1)) sr[4 * i + e] = __float_as_uint(-INFINITY);
  }

  const uint64_t c2 = f2_splat(p.scale_log2);
  uint32_t pk[16], dk[16];  // [2i + r]: row g + 8r, columns 8i + q2, 8i + q2 + 1 (16x128b)
  const int st = g % Cfg::STAGES;
  const float* vec = reinterpret_cast<const float*>(smem + Cfg::kVecOff + st * Cfg::kVecBytes);
  if (Cfg::kDKV) {
    // the L2 / D slices came by bulk copy: observe their completion before reading them (the
    // stage cannot be refilled before this step's OpFull)
    if (!wait_warp(bar(Cfg::kBarStrFull + st), static_cast<uint32_t>(g / Cfg::STAGES) & 1u, wd,
                   kSiteSoftStage))
      return false;
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int i = k >> 1, r = k & 1;
    uint64_t nl, d2;
    if (Cfg::kDKV) {
      const float2 lv = *reinterpret_cast<const float2*>(vec + 8 * i + q2);
      const float2 dv = *reinterpret_cast<const float2*>(vec + Cfg::kCols + 8 * i + q2);
      nl = f2_pack(-lv.x, -lv.y);
      d2 = f2_pack(dv.x, dv.y);
    } else {
      nl = f2_splat(-lrow[r]);
      d2 = f2_splat(drow[r]);
    }
    const uint64_t x = f2_fma(f2_pack(f(sr[2 * k]), f(sr[2 * k + 1])), c2, nl);
    float x0, x1;
    f2_unpack(x, x0, x1);
    const float e0 = ex2_approx(x0), e1 = ex2_approx(x1);
    const uint64_t t = f2_add(f2_pack(f(dp[2 * k]), f(dp[2 * k + 1])), f2_neg(d2));
    const uint64_t ds = f2_mul(f2_pack(e0, e1), t);
    float ds0, ds1;
    f2_unpack(ds, ds0, ds1);
    pk[k] = pack_pair<Cfg::kBF16>(e0, e1);
    dk[k] = pack_pair<Cfg::kBF16>(ds0, ds1);
  }
  // The operand columns are free once the previous step's TS MMAs have completed.
  if (g > 0) {
    if (!wait_warp(bar(Cfg::kBarAccDone), static_cast<uint32_t>(g - 1) & 1u, wd, kSiteSoftODone))
      return false;
    tc_fence_after();
  }
  if (Cfg::kDKV) {
    tmem_st_16x128b_x8(tOp0, pk);
    tmem_st_16x128b_x8(tOp1, dk);
  } else {
    tmem_st_16x128b_x8(tOp0, dk);
  }
  tmem_wait_st();
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(bar(Cfg::kBarOpFull));
  return true;
}

template <class Cfg>
__device__ __forceinline__ void bwd_softmax_role(const BwdParams& p, uint8_t* smem, uint32_t bars,
                                                 uint32_t tmem, const Watchdog& wd) {
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int slice = (warp & 3) * 32 + ((warp >> 2) & 1) * 16;
  const int half = warp >> 3;  // columns [64 half, 64 half + 64) of a block
  const int gq = lane >> 2;
  const int q = lane & 3;
  const uint32_t lb = static_cast<uint32_t>(slice) << 16;
  const uint32_t tS = tmem + lb + Cfg::kColS + 64 * half;
  const uint32_t tDP = tmem + lb + Cfg::kColDP + 64 * half;
  // P / dS operands: fp16 / bf16 pairs, 32 columns per half
  const uint32_t tOp0 = tmem + lb + Cfg::kColOp0 + 32 * half;
  const uint32_t tOp1 = tmem + lb + Cfg::kColOp1 + 32 * half;
  int g = 0;
  BwdCursor<Cfg> cur;
  cur.init(p);
  while (cur.valid()) {
    const int blk = cur.u % p.blocks;
    const int bh = cur.u / p.blocks;
    const int row0 = blk * Cfg::kRows + slice;  // first resident row of this warp
    float lrow[2] = {0.f, 0.f}, drow[2] = {0.f, 0.f};
    if (!Cfg::kDKV) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const size_t idx = static_cast<size_t>(bh) * p.blocks * Cfg::kRows + row0 + gq + 8 * r;
        lrow[r] = p.lse2[idx];
        drow[r] = p.di[idx];
      }
    }
    const int j0 = cur.j0, j1 = cur.j1, b = cur.seg & 1;
    for (int j = j0; j < j1; ++j, ++g) {
      if (!bwd_step<Cfg>(p, smem, bars, tS, tDP, tOp0, tOp1, lane, half, g, blk, j, row0, lrow,
                         drow, wd))
        return;
    }
    // ---- unit epilogue: accumulators -> (scaled) fp16 / bf16 -> staging -> TMA
    if (!wait_warp(bar(Cfg::kBarAccDone), static_cast<uint32_t>(g - 1) & 1u, wd, kSiteSoftOFinal))
      return;
    tc_fence_after();
    uint8_t* res = smem + Cfg::kResOff + b * 2 * Cfg::kTileBytes;
    // this warp's 32 of the 64 accumulator columns (its column half), 16-byte chunks
    // 4 half .. 4 half + 3 of each of its rows in the 128B-swizzled staging tile
    auto stage_acc = [&](uint32_t col, float mul, uint8_t* dst_tile) {
      uint32_t a[16];
      tmem_ld_16x256b_sync(tmem + lb + col + 32 * half, a);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = slice + gq + 8 * r;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t w = pack_pair<Cfg::kBF16>(__uint_as_float(a[4 * i + 2 * r]) * mul,
                                                   __uint_as_float(a[4 * i + 2 * r + 1]) * mul);
          const int chunk = 4 * half + i;
          const uint32_t dst =
              smem_addr(dst_tile + row * 128 + ((chunk ^ (row & 7)) << 4) + 4 * q);
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(dst), "r"(w) : "memory");
        }
      }
    };
    if (Cfg::kDKV) {
      stage_acc(Cfg::kColAcc1, p.scale, res);                    // dK over the k tile
      stage_acc(Cfg::kColAcc0, 1.0f, res + Cfg::kTileBytes);     // dV over the v tile
    } else {
      stage_acc(Cfg::kColAcc0, p.scale, res);                    // dQ over the q tile
    }
    tc_fence_before();
    fence_proxy_async_smem();
    __syncwarp();
    // staging rows written: the store warp takes the unit from here (bwd_store_role)
    if (lane == 0) mbar_arrive(bar(Cfg::kBarStage));
    cur.j = cur.j1 - 1;
    cur.step(p);
  }
}

// One thread of the store warp: once the 16 softmax-side warps have staged a unit's gradients
// in its resident buffers, store them with TMA and free the buffers for the load warp when
// the stores have read them; the softmax-side warps go straight on to the next unit.
template <class Cfg>
__device__ __forceinline__ void bwd_store_role(const BwdParams& p, uint8_t* smem, uint32_t bars,
                                               const Watchdog& wd) {
  auto bar = [&](int idx) { return bars + 8u * static_cast<uint32_t>(idx); };
  BwdCursor<Cfg> cur;
  cur.init(p);
  int stores = 0;
  while (cur.valid()) {
    const int b = cur.seg & 1;
    if (!wait_single(bar(Cfg::kBarStage), static_cast<uint32_t>(stores) & 1u, wd, kSiteSoftStage))
      break;
    uint8_t* res = smem + Cfg::kResOff + b * 2 * Cfg::kTileBytes;
    const int r0 = (cur.u % p.blocks) * Cfg::kRows;
    const HeadBatch hb = bwd_head_batch(p, cur.u);
    tma_store_4d(&p.tm_o0, smem_addr(res), 0, r0, hb.h, hb.b);
    if (Cfg::kDKV) tma_store_4d(&p.tm_o1, smem_addr(res + Cfg::kTileBytes), 0, r0, hb.h, hb.b);
    tma_store_commit();
    tma_store_wait_read();
    mbar_arrive(bar(Cfg::kBarResEmpty + b));
    ++stores;
    cur.j = cur.j1 - 1;
    cur.step(p);
  }
  // unwinding or done: shared memory must outlive every store's read of it
  tma_store_wait_read();
}

// The barriers of a CTA, initialised by one thread (the indices are those of both passes).
template <class Cfg>
__device__ __forceinline__ void bwd_init_bars(uint32_t bars) {
  for (int b = 0; b < 2; ++b) {
    mbar_init(bars + 8 * (Cfg::kBarResFull + b), 1);
    mbar_init(bars + 8 * (Cfg::kBarResEmpty + b), 1);
  }
  for (int s = 0; s < Cfg::STAGES; ++s) {
    mbar_init(bars + 8 * (Cfg::kBarStrFull + s), 1);
    mbar_init(bars + 8 * (Cfg::kBarStrEmpty + s), 2);  // both MMA issuers read the stage
  }
  mbar_init(bars + 8 * Cfg::kBarSSFull, 1);
  mbar_init(bars + 8 * Cfg::kBarSSFree, Cfg::kSoftmaxWarps);
  mbar_init(bars + 8 * Cfg::kBarOpFull, Cfg::kSoftmaxWarps);
  mbar_init(bars + 8 * Cfg::kBarAccDone, 1);
  mbar_init(bars + 8 * Cfg::kBarStage, Cfg::kSoftmaxWarps);
  mbar_init(bars + 8 * Cfg::kBarDrain, 1);
  mbar_init(bars + 8 * (Cfg::kBarDrain + 1), 1);
  mbar_init_fence();
}

// One CTA: the units of pass CA (params pa), then, if kTwo, those of pass CB (params pb). Between
// the passes every role has finished (the MMA warp drains its commits, the store thread waits
// for its stores' shared-memory reads), the CTA meets on named barrier 2 and the barriers
// start afresh; TMEM stays allocated. The barriers live past both passes' shared-memory
// layouts. Each role's calls stay inside its setmaxnreg branch, which is what lets the
// register allocator give the softmax-side warps their 104 registers.
template <class CA, class CB, bool kTwo>
__device__ __forceinline__ void bwd_cta(const BwdParams& pa, const BwdParams& pb) {
  static_assert(CA::kNumBars == CB::kNumBars && CA::kThreads == CB::kThreads &&
                    CA::kTmemCols == CB::kTmemCols,
                "passes of one CTA share barriers, threads and TMEM");
  constexpr int kBarOff = CA::kBarOff > CB::kBarOff ? CA::kBarOff : CB::kBarOff;
  constexpr int kTmemSlotOff = kBarOff + CA::kNumBars * 8;
  constexpr int kAbortOff = kTmemSlotOff + 4;
  static_assert(kAbortOff + 4 + 1024 <= (CA::kSmemBytes > CB::kSmemBytes ? CA::kSmemBytes
                                                                         : CB::kSmemBytes),
                "barriers inside the launch's shared memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t bars = smem_addr(smem + kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kTmemSlotOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kAbortOff);
  // Between the passes: true if the second pass runs (the same verdict in every thread:
  // nothing writes the flag between the two barriers).
  auto next_pass = [&]() -> bool {
    __syncwarp();
    tc_fence_before();
    named_bar_sync(2, CA::kThreads);
    tc_fence_after();
    const bool go = *abort_flag == 0;
    if (go && warp == CA::kLoadWarp && lane == 0) {
      for (int i = 0; i < CA::kNumBars; ++i) mbar_inval(bars + 8 * i);
      bwd_init_bars<CB>(bars);
    }
    named_bar_sync(2, CA::kThreads);
    return go;
  };
  // As in the forward kernel: the load thread initialises the barriers and goes straight on
  // to its first copies; the other warps wait on named barrier 1 for the barriers and warp
  // 0's TMEM allocation (the load warp only arrives there).
  uint32_t tmem = 0;
  if (warp == CA::kLoadWarp) {
    if (lane == 0) {
      *abort_flag = 0;
      bwd_init_bars<CA>(bars);
    }
    __syncwarp();
    named_bar_arrive(1, CA::kThreads);
    setmaxnreg_dec<CA::kControlRegs>();
    const Watchdog wd{abort_flag, pa.status, pa.timeout_ns};
    if (lane == 0) bwd_load_role<CA>(pa, smem, bars, wd);
    if constexpr (kTwo) {
      if (next_pass() && lane == 0) bwd_load_role<CB>(pb, smem, bars, wd);
    }
  } else {
    if (warp == 0) {
      tmem_alloc(smem_addr(tmem_slot), CA::kTmemCols);
      tmem_relinquish();
    }
    tc_fence_before();
    named_bar_sync(1, CA::kThreads);
    tc_fence_after();
    tmem = *tmem_slot;
    const Watchdog wd{abort_flag, pa.status, pa.timeout_ns};
    if (warp < CA::kSoftmaxWarps) {
      setmaxnreg_inc<CA::kSoftmaxRegs>();
      bwd_softmax_role<CA>(pa, smem, bars, tmem, wd);
      if constexpr (kTwo) {
        if (next_pass()) bwd_softmax_role<CB>(pb, smem, bars, tmem, wd);
      }
    } else {
      setmaxnreg_dec<CA::kControlRegs>();
      if (warp == CA::kMmaWarp) {
        bwd_mma_role<CA, false>(pa, smem, bars, tmem, wd);
      } else if (warp == CA::kAccWarp) {
        bwd_mma_role<CA, true>(pa, smem, bars, tmem, wd);
      } else if (warp == CA::kStoreWarp) {
        if (lane == 0) bwd_store_role<CA>(pa, smem, bars, wd);
      }
      if constexpr (kTwo) {
        if (next_pass()) {
          if (warp == CB::kMmaWarp) {
            bwd_mma_role<CB, false>(pb, smem, bars, tmem, wd);
          } else if (warp == CB::kAccWarp) {
            bwd_mma_role<CB, true>(pb, smem, bars, tmem, wd);
          } else if (warp == CB::kStoreWarp) {
            if (lane == 0) bwd_store_role<CB>(pb, smem, bars, wd);
          }
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, CA::kTmemCols);
}

// Both passes in one launch, at the same time on separate SMs: CTAs [0, pkv.cta0) run the dQ
// pass, the rest the dK/dV pass. Used when each pass has fewer units than about two per SM.
template <bool kCausal, bool kBF16>
__global__ void __launch_bounds__(BwdConfig<true, kCausal, kBF16>::kThreads, 1)
    mfa_bwd_kernel(const __grid_constant__ BwdParams pq, const __grid_constant__ BwdParams pkv) {
  using CQ = BwdConfig<false, kCausal, kBF16>;
  using CK = BwdConfig<true, kCausal, kBF16>;
  if (static_cast<int>(blockIdx.x) < pkv.cta0)
    bwd_cta<CQ, CQ, false>(pq, pq);
  else
    bwd_cta<CK, CK, false>(pkv, pkv);
}

// Both passes in one launch, every CTA on both: its dK/dV units first, then its dQ units,
// dealt from the other end of the grid (pq.reverse), so that the CTAs with one dK/dV unit
// more than the others have none of the extra dQ units. Used when a pass has a few units
// per SM: 512 units per pass on 148 SMs take 4 dK/dV + 3 dQ units on the slowest CTA, where
// separate SMs per pass take 7 dK/dV units (a dK/dV step costs more than a dQ step).
template <bool kCausal, bool kBF16>
__global__ void __launch_bounds__(BwdConfig<true, kCausal, kBF16>::kThreads, 1)
    mfa_bwd_mixed_kernel(const __grid_constant__ BwdParams pq,
                         const __grid_constant__ BwdParams pkv) {
  bwd_cta<BwdConfig<true, kCausal, kBF16>, BwdConfig<false, kCausal, kBF16>, true>(pkv, pq);
}

// One pass per launch (many units per SM), all CTAs on it; a kernel of its own, which measured
// 2-5% faster than the two-pass kernel above run with all CTAs on one pass.
template <bool kDKV, bool kCausal, bool kBF16>
__global__ void __launch_bounds__(BwdConfig<kDKV, kCausal, kBF16>::kThreads, 1)
    mfa_bwd_pass_kernel(const __grid_constant__ BwdParams p) {
  using C = BwdConfig<kDKV, kCausal, kBF16>;
  bwd_cta<C, C, false>(p, p);
}

// Dynamic shared memory of the two-pass launch.
template <bool kCausal, bool kBF16>
constexpr int bwd_smem_bytes() {
  return BwdConfig<false, kCausal, kBF16>::kSmemBytes > BwdConfig<true, kCausal, kBF16>::kSmemBytes
             ? BwdConfig<false, kCausal, kBF16>::kSmemBytes
             : BwdConfig<true, kCausal, kBF16>::kSmemBytes;
}

// D_i = rowsum(dO ⊙ o) and L2_i = L_i * log2(e) for every row, into [bh][blocks * 128] arrays
// padded past N with D = 0, L2 = +inf (so that padded queries get P = 0 in the dK/dV pass).
// Eight threads per row (16 bytes each), grid-stride.
template <bool kBF16>
__global__ void __launch_bounds__(256) mfa_bwd_prep_kernel(const void* o, const void* dout,
                                                           const float* lse, float* lse2,
                                                           float* di, int bh, int n, int heads,
                                                           long long stride_b, long long stride_h,
                                                           long long stride_n, int blocks) {
  const long long rows = static_cast<long long>(bh) * blocks * 128;  // a multiple of 4
  const int sub = threadIdx.x & 7;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  // four rows per warp and iteration; the trip count is the same for the whole warp
  for (long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
       w * 4 < rows; w += warps) {
    const long long r = w * 4 + ((threadIdx.x & 31) >> 3);
    const int h = static_cast<int>(r / (static_cast<long long>(blocks) * 128));
    const int row = static_cast<int>(r - static_cast<long long>(h) * blocks * 128);
    float acc = 0.0f;
    if (row < n) {
      const long long off = static_cast<long long>(h / heads) * stride_b +
                            static_cast<long long>(h % heads) * stride_h +
                            static_cast<long long>(row) * stride_n + 8 * sub;
      const uint4 a = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(o) + off);
      const uint4 b = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(dout) + off);
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float a0, a1, b0, b1;
        unpack_pair<kBF16>(aw[e], a0, a1);
        unpack_pair<kBF16>(bw[e], b0, b1);
        acc = fmaf(a0, b0, fmaf(a1, b1, acc));
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    if (sub == 0) {
      di[r] = row < n ? acc : 0.0f;
      lse2[r] = row < n ? lse[static_cast<long long>(h) * n + row] * 1.4426950408889634f
                        : INFINITY;
    }
  }
}

}  // namespace mfa
