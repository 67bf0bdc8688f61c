// e4m3 conversion and stochastic-rounding helpers shared by the quantiser
// kernels and the fused MoE dispatch (same numerics in both places).
//
// Stochastic rounding: y is written as down + frac * ulp with ulp the e4m3
// spacing at |y| (2^(e-3) for normal values, 2^-9 below 2^-6), and rounds up
// with probability frac. Random bits come from the "lowbias32" integer hash
// (C. Wellons, public domain) of (seed, element index).
#pragma once

#include <cuda_fp8.h>
#include <stdint.h>

namespace ntb {

__device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352dU;
  x ^= x >> 15;
  x *= 0x846ca68bU;
  x ^= x >> 16;
  return x;
}

__device__ __forceinline__ float uniform01(uint64_t seed, uint64_t idx) {
  const uint32_t h = lowbias32(static_cast<uint32_t>(idx) ^ lowbias32(static_cast<uint32_t>(seed) ^
                                                                     lowbias32(static_cast<uint32_t>(idx >> 32) +
                                                                               static_cast<uint32_t>(seed >> 32))));
  return (h >> 8) * (1.0f / 16777216.0f);
}

// Stochastic rounding of y (|y| <= 448) onto the e4m3 grid, by exponent arithmetic: the grid
// spacing at |y| is ulp = 2^(floor(log2|y|) - 3) (2^-9 below 2^-6, the subnormal spacing), a power
// of two built from y's exponent field, so t = |y| / ulp is exact and floor(t + u) rounds |y| up to
// the next grid point with probability frac(t). The sign is applied afterwards.
__device__ __forceinline__ float e4m3_sr(float y, float u) {
  const int e = static_cast<int>((__float_as_uint(y) >> 23) & 0xFFu) - 127;  // floor(log2|y|) (normal y)
  const int ex = (e < -6 ? -6 : e) - 3;                                       // log2 of the spacing
  const float inv_ulp = __uint_as_float(static_cast<uint32_t>(127 - ex) << 23);
  const float ulp = __uint_as_float(static_cast<uint32_t>(127 + ex) << 23);
  const float r = floorf(fmaf(fabsf(y), inv_ulp, u)) * ulp;
  return copysignf(fminf(r, 448.f), y);
}

// x / s rounded to nearest in fp32 from one reciprocal per scale: y = RN(1/s), q0 = RN(x y),
// r = x - s q0 (exact with an FMA), q = RN(q0 + r y). This is the FMA division correction of
// P. Markstein (IBM J. Res. Dev. 34(1), 1990; Muller et al., Handbook of Floating-Point Arithmetic,
// Markstein's theorem): with y within half an ulp of 1/s and q0 within one ulp of x / s, q is the
// correctly rounded quotient, provided no intermediate underflows. A quotient below 2^-126 may
// differ in its last bit; it rounds to 0 in e4m3 either way (smallest e4m3 subnormal 2^-9). Scales
// whose reciprocal is not a normal number take the IEEE division.
struct ScaleDiv {
  float s, y;
  bool fast;
};

__device__ __forceinline__ ScaleDiv make_scale_div(float s) {
  const float y = __frcp_rn(s);
  const bool fast = s >= 1.17549435e-38f && s <= 8.50705917e37f && y >= 1.17549435e-38f;
  return {s, y, fast};
}

__device__ __forceinline__ float div_scale(float x, const ScaleDiv& d) {
  if (!d.fast) return __fdiv_rn(x, d.s);
  const float q0 = __fmul_rn(x, d.y);
  const float r = fmaf(-d.s, q0, x);
  return fmaf(r, d.y, q0);
}

__device__ __forceinline__ uint8_t to_e4m3(float y) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3));
}

// Two values to two e4m3 codes in one conversion (saturating, round to nearest even): a in the
// low byte.
__device__ __forceinline__ uint32_t to_e4m3x2(float a, float b) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3)) & 0xFFFFu;
}

__device__ __forceinline__ float from_e4m3(uint8_t q) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(q), __NV_E4M3);
  return __half2float(__half(h));
}

}  // namespace ntb
