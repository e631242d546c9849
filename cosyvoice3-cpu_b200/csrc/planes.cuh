// Activation planes: the operand format of cv3_tc_gemm_q8_planes.
//
// An fp32 activation matrix X[M][K] (K a multiple of 64) is stored as
//   planes fp16 [M][2K]: for row m and 64-wide group g, the 64 values
//          hi = fp16(x * 2^e) at [m][128 g .. 128 g + 63] and
//          lo = fp16(x * 2^e - hi) at [m][128 g + 64 .. 128 g + 127];
//   exps   int8 [K/64][lde] (lde >= M, a multiple of 16): e for (g, m),
// where e brings the group's largest |x| into [2^14, 2^15).  hi + lo carries 22
// significant bits of every value (the power-of-two scaling is exact), the
// precision the 3xTF32 split gives an fp32 operand; the planes take the fp32
// matrix's bytes, and the GEMM reads them by TMA with no conversion step.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace cv3p {

// the exponent e with max|x| * 2^e in [2^14, 2^15), clamped to [-126, 126]
__device__ __forceinline__ int group_exponent(float amax) {
  if (!(amax > 0.f)) return 0;
  const int e = ((__float_as_int(amax) >> 23) & 0xFF) - 127;
  const int s = 14 - e;
  return s > 126 ? 126 : (s < -126 ? -126 : s);
}

// 2^e as a float, e in [-126, 127]
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// (a0, a1) (already scaled) -> hi and lo half2 words, a0 in the low halves
__device__ __forceinline__ void split_pair(float a0, float a1, uint32_t& hi, uint32_t& lo) {
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(a1), "f"(a0));
  __half2 h = *reinterpret_cast<__half2*>(&hi);
  const float r0 = a0 - __low2float(h), r1 = a1 - __high2float(h);
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(r1), "f"(r0));
}

}  // namespace cv3p
