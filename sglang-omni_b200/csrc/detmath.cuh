// Deterministic exp shared by the sampling and routing kernels and the CPU
// oracle (bit-exact parity): Cody–Waite range reduction by ln 2 split into a
// high part with trailing zero bits and a low correction, then the degree-7
// Taylor polynomial of e^r in Horner form with explicit round-to-nearest
// multiply-adds, and an exact power-of-two scaling.
#pragma once
#include "common.cuh"

namespace omni {
OMNI_DEVINL float scale_pow2_f(float p, int n) {
  if (n > 127) {
    p = __fmul_rn(p, __uint_as_float(0x7F000000u));
    n -= 127;
    if (n > 127) n = 127;
  }
  if (n < -126) {
    p = __fmul_rn(p, __uint_as_float(0x00800000u));
    n += 126;
    if (n < -126) n = -126;
  }
  return __fmul_rn(p, __uint_as_float((uint32_t)(n + 127) << 23));
}

OMNI_DEVINL float det_expf(float x) {
  if (x != x) return x;
  if (x > 88.7228394f) return __uint_as_float(0x7F800000u);
  if (x < -103.972084f) return 0.0f;
  float t = __fmul_rn(x, 0x1.715476p+0f);
  float n = floorf(__fadd_rn(t, 0.5f));
  float r = __fmaf_rn(-n, 0x1.62e4p-1f, x);
  r = __fmaf_rn(-n, 0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
  p = __fmaf_rn(p, r, 0x1.111112p-7f);
  p = __fmaf_rn(p, r, 0x1.555556p-5f);
  p = __fmaf_rn(p, r, 0x1.555556p-3f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  return scale_pow2_f(p, (int)n);
}

}  // namespace omni
