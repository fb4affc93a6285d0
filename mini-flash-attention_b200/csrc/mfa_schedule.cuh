// Work schedule of the attention forward, shared by the launcher (host), the forward kernel
// and the merge kernel (device).
//
// A step is one key block (128 keys) of one query block (rows_per_unit query rows) of one
// (batch * head) row; a unit is one query block of one head, u = head * q_blocks + qb. Steps
// are numbered head-major and, within a head, query block by query block in the head's
// processing order, key blocks ascending. Without causal masking every query block has
// nkb = ceil(N / 128) steps and the order is qb = 0, 1, 2, ... With causal masking (key
// index > query index masked, as the reference's test and benchmark build the mask,
// tests/test_forward.py:30-32 and benchs/benchmark_forward.py:109-112) query block qb needs
// only the key blocks that start at or before its last row: group * (qb + 1) with group =
// rows_per_unit / 128, nkb for the last block. Its order pairs short and long blocks,
// qb = 0, Q-1, 1, Q-2, ... (Q = q_blocks): every pair after the first has group * (Q + 1)
// steps, so an even split of the steps gives every CTA about the same number of query
// blocks, i.e. of unit epilogues and diagonal (masked) blocks, and a step is located in O(1).
// A launch over a range of query rows that starts at query block qb0 of the head (a row range
// that begins on a unit boundary) numbers its blocks from there: block qb needs
// group * (qb + 1 + qb0) key blocks, and the pairs keep a constant length.
#pragma once

#include <cmath>
#include <cstdint>

namespace mfa {

// n / d for 0 <= n < 2^31 as (n * mul) >> shift: shift = 31 + ceil(log2 d) and
// mul = ceil(2^shift / d) < 2^32, so the error of n * mul / 2^shift stays below
// 2^-ceil(log2 d) <= 1/d. The kernels split step and unit indices with it where a division
// by a runtime value would cost ~20 (32-bit) or ~100 (64-bit) instructions.
struct Div31 {
  uint32_t mul;
  int shift;
  void set(long long d) {
    int lg = 0;
    while ((1LL << lg) < d) ++lg;
    shift = 31 + lg;
    mul = static_cast<uint32_t>(((uint64_t{1} << shift) + static_cast<uint64_t>(d) - 1) /
                                static_cast<uint64_t>(d));
  }
  __host__ __device__ uint32_t operator()(uint32_t n) const {
    return static_cast<uint32_t>((static_cast<uint64_t>(n) * mul) >> shift);
  }
};

struct Schedule {
  int bh;                // batch * heads
  int q_blocks;          // query blocks per head: ceil(N / rows_per_unit)
  int nkb;               // key blocks per head: ceil(N / 128)
  int group;             // rows_per_unit / 128
  int causal;            // 1: query block qb stops at key block group * (qb + 1 + qb0)
  int qb0;               // causal: query blocks of the head before this launch's first
  long long head_steps;  // steps of one head
  // split mode: CTA c of `ctas` takes the global steps [c * total / ctas, (c+1) * total / ctas),
  // computed as c * cta_q + c * cta_r / ctas with total = cta_q * ctas + cta_r (set_ctas)
  int ctas;
  int cta_r;
  long long cta_q;
  Div31 qdiv;  // by q_blocks (unit -> head)
  Div31 kdiv;  // by nkb (step -> unit, non-causal), for steps < 2^31
  Div31 hdiv;  // by head_steps (step -> head, causal), if head_steps < 2^31
  Div31 pdiv;  // by pair_steps() (causal locate within a head)

  __host__ __device__ int head_of(int u) const { return static_cast<int>(qdiv(u)); }
  __host__ __device__ int qb_of(int u) const { return u - head_of(u) * q_blocks; }

  // Steps [begin, end) of CTA `cta` in split mode.
  __host__ __device__ void range(int cta, long long& begin, long long& end) const {
    // cta_r * cta < ctas^2 < 2^32 (ctas <= 65535, checked by set_ctas)
    const auto part = [&](int c) {
      return cta_q * c + static_cast<long long>(static_cast<uint32_t>(cta_r) *
                                                static_cast<uint32_t>(c) /
                                                static_cast<uint32_t>(ctas));
    };
    begin = part(cta);
    end = part(cta + 1);
  }

  // The kernels use the forms with the masking mode as a compile-time argument (kCausal must
  // equal `causal`), so that the non-causal kernels carry none of the causal arithmetic.
  template <bool kCausal>
  __host__ __device__ int steps_of(int qb) const {
    if (!kCausal) return nkb;
    // only the last query block can reach past key block nkb - 1 (it holds row N - 1)
    return qb == q_blocks - 1 ? nkb : (qb + 1 + qb0) * group;
  }
  // Causal order: query block at position k of its head, and the position of query block qb.
  __host__ __device__ int qb_at(int k) const {
    return (k & 1) ? q_blocks - 1 - (k >> 1) : (k >> 1);
  }
  __host__ __device__ int pos_of(int qb) const {
    return 2 * qb < q_blocks ? 2 * qb : 2 * (q_blocks - 1 - qb) + 1;
  }
  // Causal: steps of the first pair (query blocks 0 and Q-1) and of every later pair.
  __host__ __device__ long long pair0() const {
    return static_cast<long long>(group) * (1 + qb0) + nkb;
  }
  __host__ __device__ long long pair_steps() const {
    return static_cast<long long>(group) * (q_blocks + 1 + 2LL * qb0);
  }
  // Causal: first step (within its head) of the query block at position k.
  __host__ __device__ long long pos_first(int k) const {
    const int m = k >> 1;
    long long f = m == 0 ? 0 : pair0() + (m - 1) * pair_steps();
    if (k & 1) f += steps_of<true>(m);
    return f;
  }
  // First step of query block qb inside its head.
  template <bool kCausal>
  __host__ __device__ long long first_of(int qb) const {
    return kCausal ? pos_first(pos_of(qb)) : static_cast<long long>(qb) * nkb;
  }
  __host__ __device__ long long total() const { return head_steps * bh; }
  // First global step of unit u.
  template <bool kCausal>
  __host__ __device__ long long unit_first(int u) const {
    return static_cast<long long>(head_of(u)) * head_steps + first_of<kCausal>(qb_of(u));
  }
  // The unit processed after unit u (in split mode, where a CTA walks consecutive steps).
  template <bool kCausal>
  __host__ __device__ int next_unit(int u) const {
    if (!kCausal) return u + 1;
    const int head = head_of(u);
    const int k = pos_of(u - head * q_blocks) + 1;
    return k < q_blocks ? head * q_blocks + qb_at(k) : (head + 1) * q_blocks;
  }
  // Unit u and key block j of global step s (0 <= s < total()).
  template <bool kCausal>
  __host__ __device__ void locate(long long s, int& u, int& j) const {
    const bool small = s < (1LL << 31);
    if (!kCausal) {  // every query block has nkb steps
      const long long uu = small ? static_cast<long long>(kdiv(static_cast<uint32_t>(s))) : s / nkb;
      u = static_cast<int>(uu);
      j = static_cast<int>(s - uu * nkb);
      return;
    }
    const long long head = small && head_steps < (1LL << 31)
                               ? static_cast<long long>(hdiv(static_cast<uint32_t>(s)))
                               : s / head_steps;
    const long long r = s - head * head_steps;
    const int pairs = q_blocks >> 1;
    int k;
    long long rem;
    if (pairs > 0 && r < pair0()) {
      k = 0;
      rem = r;
    } else if (pairs > 1 && r < pair0() + (pairs - 1) * pair_steps()) {
      const long long t = r - pair0();  // < head_steps; pair_steps() < 2^31 (see set_ctas)
      const long long m =
          1 + (t < (1LL << 31) ? static_cast<long long>(pdiv(static_cast<uint32_t>(t)))
                               : t / pair_steps());
      k = static_cast<int>(2 * m);
      rem = t - (m - 1) * pair_steps();
    } else {  // the middle query block of an odd count, alone at the last position
      k = q_blocks - 1;
      rem = r - pos_first(k);
    }
    if (!(k & 1) && k + 1 < q_blocks) {  // a pair: the short block, then the long one
      const int s_even = steps_of<true>(k >> 1);
      if (rem >= s_even) {
        ++k;
        rem -= s_even;
      }
    }
    u = static_cast<int>(head * q_blocks + qb_at(k));
    j = static_cast<int>(rem);
  }
};

// nq query rows and nk keys per head. Causal: the rows start at query block qb0 of the head
// and nk is one past their last row (the keys after it are masked for every row).
inline Schedule make_schedule(long long bh, long long nq, long long nk, int rows_per_unit,
                              int keys_per_block, bool causal, int qb0 = 0) {
  Schedule s;
  s.bh = static_cast<int>(bh);
  s.qb0 = causal ? qb0 : 0;
  s.q_blocks = static_cast<int>((nq + rows_per_unit - 1) / rows_per_unit);
  s.nkb = static_cast<int>((nk + keys_per_block - 1) / keys_per_block);
  s.group = rows_per_unit / keys_per_block;
  s.causal = causal ? 1 : 0;
  s.head_steps = causal ? s.pos_first(s.q_blocks - 1) + s.steps_of<true>(s.qb_at(s.q_blocks - 1))
                       : s.first_of<false>(s.q_blocks - 1) + s.steps_of<false>(s.q_blocks - 1);
  s.qdiv.set(s.q_blocks);
  s.kdiv.set(s.nkb);
  s.hdiv.set(s.head_steps < (1LL << 31) ? s.head_steps : 1);
  s.pdiv.set(s.pair_steps());
  s.ctas = 1;
  s.cta_q = s.total();
  s.cta_r = 0;
  return s;
}

// Split mode over `ctas` CTAs (1 <= ctas <= 65535).
inline void set_ctas(Schedule& s, int ctas) {
  s.ctas = ctas;
  s.cta_q = s.total() / ctas;
  s.cta_r = static_cast<int>(s.total() % ctas);
}

}  // namespace mfa
