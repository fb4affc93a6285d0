// Work schedule of the attention forward, shared by the launcher (host), the forward kernel
// and the merge kernel (device).
//
// A step is one key block (128 keys) of one query block (rows_per_unit query rows) of one
// (batch * head) row. Steps are numbered row-major over (head, query block, key block). Without
// causal masking every query block has nkb = ceil(N / 128) steps. With causal masking (key
// index > query index masked, as the reference's test and benchmark build the mask,
// tests/test_forward.py:30-32 and benchs/benchmark_forward.py:109-112) query block qb needs
// only the key blocks that start at or before its last row: min(nkb, group * (qb + 1)) with
// group = rows_per_unit / 128, so a head's steps form a triangle and a step's query block is
// found from the inverse triangular number.
#pragma once

#include <cmath>
#include <cstdint>

namespace mfa {

struct Schedule {
  int bh;                // batch * heads
  int q_blocks;          // query blocks per head: ceil(N / rows_per_unit)
  int nkb;               // key blocks per head: ceil(N / 128)
  int group;             // rows_per_unit / 128
  int causal;            // 1: query block qb stops at key block group * (qb + 1)
  long long head_steps;  // steps of one head

  // The kernels use the forms with the masking mode as a compile-time argument (kCausal must
  // equal `causal`), so that the non-causal kernels carry none of the causal arithmetic.
  template <bool kCausal>
  __host__ __device__ int steps_of(int qb) const {
    if (!kCausal) return nkb;
    const int need = (qb + 1) * group;
    return need < nkb ? need : nkb;
  }
  // First step of query block qb inside its head. Only the last query block can be capped by
  // nkb (every earlier block ends before row N), so the triangular sum is exact for all qb.
  template <bool kCausal>
  __host__ __device__ long long first_of(int qb) const {
    return kCausal ? static_cast<long long>(group) * qb * (qb + 1) / 2
                   : static_cast<long long>(qb) * nkb;
  }
  __host__ __device__ long long total() const { return head_steps * bh; }
  // First global step of unit u (row-major over (head, query block)).
  template <bool kCausal>
  __host__ __device__ long long unit_first(int u) const {
    return static_cast<long long>(u / q_blocks) * head_steps + first_of<kCausal>(u % q_blocks);
  }
  // Unit u and key block j of global step s (0 <= s < total()).
  template <bool kCausal>
  __host__ __device__ void locate(long long s, int& u, int& j) const {
    if (!kCausal) {  // every query block has nkb steps
      const long long uu = s / nkb;
      u = static_cast<int>(uu);
      j = static_cast<int>(s - uu * nkb);
      return;
    }
    const long long head = s / head_steps;
    const long long r = s - head * head_steps;
    int qb;
    {
      // largest qb with group * qb * (qb + 1) / 2 <= r, from the float root and corrected
      qb = static_cast<int>((sqrtf(8.0f * static_cast<float>(r) / group + 1.0f) - 1.0f) * 0.5f);
      if (qb > q_blocks - 1) qb = q_blocks - 1;
      if (qb < 0) qb = 0;
      while (qb + 1 < q_blocks && first_of<kCausal>(qb + 1) <= r) ++qb;
      while (qb > 0 && first_of<kCausal>(qb) > r) --qb;
    }
    u = static_cast<int>(head * q_blocks + qb);
    j = static_cast<int>(r - first_of<kCausal>(qb));
  }
};

inline Schedule make_schedule(long long bh, long long n, int rows_per_unit, int keys_per_block,
                              bool causal) {
  Schedule s;
  s.bh = static_cast<int>(bh);
  s.q_blocks = static_cast<int>((n + rows_per_unit - 1) / rows_per_unit);
  s.nkb = static_cast<int>((n + keys_per_block - 1) / keys_per_block);
  s.group = rows_per_unit / keys_per_block;
  s.causal = causal ? 1 : 0;
  s.head_steps = causal ? s.first_of<true>(s.q_blocks - 1) + s.steps_of<true>(s.q_blocks - 1)
                       : s.first_of<false>(s.q_blocks - 1) + s.steps_of<false>(s.q_blocks - 1);
  return s;
}

// Split-mode range of CTA `cta` of `ctas` over the global steps: [begin, end).
__host__ __device__ inline void split_range(long long total, int cta, int ctas, long long& begin,
                                            long long& end) {
  begin = total * cta / ctas;
  end = total * (cta + 1) / ctas;
}

}  // namespace mfa
