// 2^x on the FMA pipe, two values at a time, for the attention softmax.
//
// The softmax needs one exponential per score; the SM's MUFU unit does 16 of
// them per clock while the FMA pipe has spare issue slots, so part of the
// exponentials is computed here instead:
//   x = j + f,  j = rint(x) (by adding and subtracting 1.5 * 2^23),
//   2^f for f in [-0.5, 0.5] by a degree-4 polynomial whose coefficients are
//   the Remez (minimax, relative error) fit printed by exp2_poly.py, rounded
//   to fp32 (maximum relative error 2.6e-6 with exact arithmetic; the result
//   is rounded to fp16, relative step 2^-11, before it is used as P),
//   2^j by adding j to the exponent field of 2^f.
// Inputs are clamped below at -126 (the result is then about 2^-126 instead
// of a smaller value; in the softmax such a probability rounds to 0 in fp16
// and adds nothing measurable to the fp32 row sum).  Valid for x <= 127.
#pragma once
#include <cuda_runtime.h>

namespace lbrr {

__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kC0 = 0.9999992847442627f, kC1 = 0.6931217908859253f, kC2 = 0.240247443318367f,
                  kC3 = 0.05591785907745361f, kC4 = 0.009570102207362652f;
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: x + kRound rounds x to an integer
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 j = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), x);  // exact
  float2 p = __ffma2_rn(make_float2(kC4, kC4), f, make_float2(kC3, kC3));
  p = __ffma2_rn(p, f, make_float2(kC2, kC2));
  p = __ffma2_rn(p, f, make_float2(kC1, kC1));
  p = __ffma2_rn(p, f, make_float2(kC0, kC0));
  // the low bits of t hold j; shifted by 23 they land in the exponent field
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

}  // namespace lbrr
