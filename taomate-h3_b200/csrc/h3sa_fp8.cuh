// Per-head e4m3 quantisation arithmetic shared by the quantisers and the fused prologue:
// y = RTNE(clamp(x / scale, -448, 448)) with the division correctly rounded.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace h3sa {

constexpr float kFp8Max = 448.0f;

// Correctly rounded x / s from y = RN(1 / s) with two residual corrections: q0 = RN(x * y) is
// within two ulps of the quotient, one correction q1 = RN(q0 + RN(x - s * q0) * y) makes it
// faithful, after which the residual x - s * q1 is exact in an FMA and RN(q1 + r1 * y) is the
// correctly rounded quotient (Markstein's division theorem). Same results as an IEEE division
// for the normal-range quotients a per-head scale produces.
__device__ __forceinline__ float div_by_scale(float x, float s, float y) {
  const float q0 = __fmul_rn(x, y);
  const float q1 = __fmaf_rn(__fmaf_rn(-s, q0, x), y, q0);
  return __fmaf_rn(__fmaf_rn(-s, q1, x), y, q1);
}

__device__ __forceinline__ uint32_t quant4(float a, float b, float c, float d, float s, float y) {
  a = fminf(fmaxf(div_by_scale(a, s, y), -kFp8Max), kFp8Max);
  b = fminf(fmaxf(div_by_scale(b, s, y), -kFp8Max), kFp8Max);
  c = fminf(fmaxf(div_by_scale(c, s, y), -kFp8Max), kFp8Max);
  d = fminf(fmaxf(div_by_scale(d, s, y), -kFp8Max), kFp8Max);
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(b), "f"(a));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(d), "f"(c));
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

}  // namespace h3sa
