// Packed fp32 pair arithmetic (fma/add .f32x2) and a polynomial exp2 that runs on the FMA
// pipe, used to take part of the softmax exponentials off the MUFU unit (16 ex2 / clk / SM
// on B200, the bottleneck of a D=64 attention forward).
//
// exp2 emulation: 2^x = 2^j * 2^f, j = round-to-nearest(x) obtained by adding 1.5 * 2^23
// (the integer lands in the low mantissa bits), f = x - j in [-1/2, 1/2], 2^f from a degree-3
// minimax polynomial (relative error 7.5e-5, below the 2^-11 rounding of the fp16 P operand),
// and the exponent j is added into the result's exponent field with one integer add.
// Coefficients: csrc/gen_exp2_poly.py (Remez exchange on the relative error).
#pragma once

#include <cstdint>

namespace mfa {

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ uint64_t f2_splat(float x) { return f2_pack(x, x); }

__device__ __forceinline__ uint64_t f2_neg(uint64_t a) { return a ^ 0x8000000080000000ull; }

// 2^x for a pair, on the FMA pipe. Inputs below -125 are clamped (the result is then
// ~2^-125, i.e. zero for every consumer here); inputs are expected <= 2^22.
__device__ __forceinline__ void exp2_poly_pair(float x0, float x1, float& y0, float& y1) {
  constexpr float kC0 = 0.9999280571937561f;
  constexpr float kC1 = 0.6932609677314758f;
  constexpr float kC2 = 0.2426111251115799f;
  constexpr float kC3 = 0.0551716685295105f;
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const uint64_t x = f2_pack(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t t = f2_add(x, f2_splat(kRound));       // j in the low mantissa bits
  const uint64_t j = f2_add(t, f2_splat(-kRound));      // j as a float
  const uint64_t f = f2_fma(j, f2_splat(-1.0f), x);     // x - j, exact
  uint64_t p = f2_fma(f2_splat(kC3), f, f2_splat(kC2));
  p = f2_fma(p, f, f2_splat(kC1));
  p = f2_fma(p, f, f2_splat(kC0));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  // (t_bits << 23) == j << 23 (mod 2^32): the 0x4B400000 bias shifts out of the word.
  y0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  y1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

}  // namespace mfa
