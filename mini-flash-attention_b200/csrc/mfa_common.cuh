// Shared pieces of the attention kernels: launch parameters, the device status codes and the
// bounded mbarrier waits (watchdog) every role uses.
#pragma once

#include <cuda.h>
#include <cstdint>

#include "mfa_ptx.cuh"
#include "mfa_schedule.cuh"

namespace mfa {

struct FwdParams {
  // {D=64, N, H, B} fp16 / bf16 views of q, k, v, out (box 64 x 128 x 1 x 1, 128B swizzle);
  // the strides carry the memory layout ([B, H, N, D] or [B, N, H, D]).
  CUtensorMap tm_q;
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  CUtensorMap tm_o;
  int n;                      // sequence length (keys, and queries of a whole launch)
  int nq;                     // query rows per head in this launch (n, or a row range's length:
                              // tm_q / tm_o then start at the range's first row)
  int q0;                     // the range's first row (0 for a whole launch): causal mask origin
  int heads;                  // H: a (batch * head) row bh is head bh % H of batch bh / H
  Schedule sc;                // query blocks, key blocks and steps (mfa_schedule.cuh)
  // Persistent schedule. split == 0 (never with causal masking): whole query blocks, CTA c
  // takes units c, c + gridDim.x, ... . split == 1: the global steps are cut into gridDim.x
  // contiguous ranges of equal length; a query block processed in pieces by several CTAs
  // leaves partial results (unnormalised O, row max, row sum) in `workspace`, which the merge
  // kernel combines.
  int split;
  float scale_log2;           // softmax scale * log2(e)
  unsigned long long timeout_ns;  // per-wait watchdog limit
  int* status;                // device status word (0 = ok)
  float* workspace;           // split mode: 2 * gridDim.x partial-result slots
  // Optional (null: not written): natural-log row log-sum-exp of the scaled scores,
  // lse[bh * N + row] = ln(sum_k exp(scale * q.k)), for the backward pass.
  float* lse;
};

// Status codes written to FwdParams::status by the watchdog: kStatusTimeoutBase + site. The
// backward kernel reports its corresponding waits under the same codes: resident tiles as
// kSiteMmaQ, streamed tiles as kSiteMmaK, S / dP read as kSiteMmaSFree / kSiteSoftSFull,
// the P / dS operands as kSiteMmaPFull, the accumulations as kSiteSoftODone / kSiteSoftOFinal,
// the streamed L / D slices and the staging as kSiteSoftStage. (11, 12 and 14 are unused.)
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
  kSiteLoadQEmpty = 13,
  kSiteSoftStage = 15,
  kSiteMmaDrain = 16,
};

// Head and batch index of a (batch * head) row.
struct HeadBatch {
  int h, b;
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

}  // namespace mfa
