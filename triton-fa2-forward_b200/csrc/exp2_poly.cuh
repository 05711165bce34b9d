// Base-2 exponential on the FMA pipe, used for a fixed subset of the softmax
// exponentials so the MUFU unit (16 ex2 / clk / SM on B200, the same rate at which the
// tensor cores consume scores at D = 128) stops being the bottleneck.
//
// Method (our own; coefficients fitted by gen_exp2_poly.py):
//   Cody-Waite range reduction  x = n + f,  n = round(x) (round-to-nearest via the
//   1.5 * 2^23 add trick), f = x - n in [-1/2, 1/2];  2^f ~= p(f), a minimax polynomial
//   in relative error found with the Remez exchange; 2^n is applied with one integer
//   multiply-add into the exponent field.  Degree 3 (max rel err 7.5e-5) is used when P
//   is rounded to bf16 (half-ulp 2e-3), degree 4 (2.7e-6) when P is rounded to fp16.
//
// Inputs are clamped to >= -125 so the exponent field never underflows; 2^-125 is far
// below anything that survives the bf16/fp16 rounding of P. The callers only use this
// on score tiles with no masked (-inf) entries, so exact zeros stay MUFU-produced.
#pragma once

#include <cstdint>
#include "ptx_sm100.cuh"

namespace fa2 {

// Coefficients c_0..c_DEG of p(f) = sum c_i f^i  (gen_exp2_poly.py output).
template <int DEG>
__device__ __forceinline__ constexpr float exp2_coef(int i) {
  if constexpr (DEG == 3) {
    return i == 0 ? 9.999280572e-01f : i == 1 ? 6.932609677e-01f : i == 2 ? 2.426111251e-01f : 5.517166853e-02f;
  } else {
    static_assert(DEG == 4, "degree 3 or 4");
    return i == 0 ? 9.999992847e-01f : i == 1 ? 6.931217909e-01f : i == 2 ? 2.402474433e-01f
         : i == 3 ? 5.591785908e-02f : 9.570102207e-03f;
  }
}

// y0 = 2^x0, y1 = 2^x1, computed as a packed pair on the FP32x2 pipe.
template <int DEG>
__device__ __forceinline__ void exp2_poly_x2(float x0, float x1, float& y0, float& y1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x0 = fmaxf(x0, -125.0f);
  x1 = fmaxf(x1, -125.0f);
  const uint64_t X = f2_pack(x0, x1);
  const uint64_t T = f2_add(X, f2_pack(kRound, kRound));        // low mantissa bits = round(x)
  const uint64_t N = f2_add(T, f2_pack(-kRound, -kRound));      // round(x) as a float (exact)
  const uint64_t F = f2_fma(N, f2_pack(-1.0f, -1.0f), X);       // f = x - n, exact
  uint64_t P = f2_pack(exp2_coef<DEG>(DEG), exp2_coef<DEG>(DEG));
#pragma unroll
  for (int i = DEG - 1; i >= 0; --i) {
    P = f2_fma(P, F, f2_pack(exp2_coef<DEG>(i), exp2_coef<DEG>(i)));
  }
  float p0, p1, t0, t1;
  f2_unpack(P, p0, p1);
  f2_unpack(T, t0, t1);
  // bits(T) = 0x4B400000 + n; (bits(T) << 23) wraps to n << 23, the exponent increment.
  y0 = __uint_as_float(__float_as_uint(t0) * 8388608u + __float_as_uint(p0));
  y1 = __uint_as_float(__float_as_uint(t1) * 8388608u + __float_as_uint(p1));
}

}  // namespace fa2
