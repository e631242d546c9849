// The snake activation of the vocoder, y = x + 1 / (alpha + 1e-9) * sin(alpha x)^2
// (cv3cpu/ops.py:77-81), with the squared sine evaluated without branches.
//
// sin_sq_fast(x), |x| <= 8192: Cody-Waite reduction r = x - k pi/2 (k = rint(2x / pi)),
// with pi/2 split into three floats P1 + P2 + P3 (P1 = pi/2 rounded, P2 and P3 the
// rounded remainders) and each step an FMA: x - k P1 is exact (for |x| >= 1 both terms
// are multiples of 2^-23 and the difference is below 1; below that k is 0 or the
// difference is exact by Sterbenz's lemma), the two later steps carry the rest of pi/2
// to ~1e-23.  On |r| <= pi/4 the Taylor series of sin to r^9 and of cos to
// r^10 truncate below 2.2e-9 relative, under a float's half ulp; the square of sin(r)
// for even k and of cos(r) for odd k is sin(x)^2 (the sign drops out).  Emulated in
// float32 over 2M arguments in [-8192, 8192] and at the floats nearest k pi/2 (k < 5000)
// and their neighbours, its absolute error is at most 1.3e-7, the same as numpy's
// float32 sin squared.
// The constants are pi/2 and the factorials' reciprocals, rounded to float.
#pragma once

namespace cv3snake {

constexpr float FAST_MAX = 8192.f;  // |x| up to which sin_sq_fast holds

__device__ __forceinline__ float sin_sq_fast(float x) {
  constexpr float P1 = 1.5707963705062866f, P2 = -4.371138828673793e-08f, P3 = -1.7151245100058819e-15f;
  constexpr float TWO_OVER_PI = 0.6366197466850281f;
  const float k = rintf(x * TWO_OVER_PI);
  float r = fmaf(-k, P1, x);
  r = fmaf(-k, P2, r);
  r = fmaf(-k, P3, r);
  const float r2 = r * r;
  // sin r = r + r^3 (-1/3! + r^2 (1/5! + r^2 (-1/7! + r^2 / 9!)))
  float ps = fmaf(r2, 2.7557318844628753e-06f, -1.9841270113829523e-04f);
  ps = fmaf(r2, ps, 8.333333767950535e-03f);
  ps = fmaf(r2, ps, -1.666666716337204e-01f);
  const float s = fmaf(r * r2, ps, r);
  // cos r = 1 + r^2 (-1/2! + r^2 (1/4! + r^2 (-1/6! + r^2 (1/8! - r^2 / 10!))))
  float pc = fmaf(r2, -2.755731998149713e-07f, 2.4801587642286904e-05f);
  pc = fmaf(r2, pc, -1.3888889225199819e-03f);
  pc = fmaf(r2, pc, 4.16666679084301e-02f);
  pc = fmaf(r2, pc, -0.5f);
  const float c = fmaf(r2, pc, 1.0f);
  const float v = (static_cast<int>(k) & 1) ? c : s;
  return v * v;
}

// sin(x)^2 for any x: the branch-free form, CUDA's sinf beyond FAST_MAX (and for inf / nan)
__device__ __forceinline__ float sin_sq(float x) {
  if (fabsf(x) <= FAST_MAX) return sin_sq_fast(x);
  const float s = sinf(x);
  return s * s;
}

// 1 / (alpha + 1e-9) rounded to nearest: rcp.rn gives the bits of the IEEE division 1.0f / d
__device__ __forceinline__ float inv_alpha(float alpha) { return __frcp_rn(alpha + 1e-9f); }

// x + inv * s2 in the reference's order: the product rounded, then the sum
__device__ __forceinline__ float snake_combine(float x, float inv, float s2) {
  return __fadd_rn(x, __fmul_rn(inv, s2));
}

}  // namespace cv3snake
