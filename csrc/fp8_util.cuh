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

__device__ __forceinline__ uint8_t to_e4m3(float y) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float from_e4m3(uint8_t q) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(q), __NV_E4M3);
  return __half2float(__half(h));
}

}  // namespace ntb
