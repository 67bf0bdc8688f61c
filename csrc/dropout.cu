// Inverted dropout for sm_100a with a counter-based generator, so the backward pass
// regenerates the mask from (seed, element index) instead of storing it.
//
// Random bits: Philox-4x32-10 (J. Salmon, M. Moraes, R. Dror, D. Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011), counter = (element index / 4 as 64 bits, 0, 0),
// key = the 64-bit seed; output word j drives element 4 * (index / 4) + j. An element is
// kept when (word >> 8) * 2^-24 >= p and then scaled by 1 / (1 - p). Forward and backward
// are the same kernel (y = x * keep * scale, dx = dy * keep * scale).
//
// Reference parity: src/layers.py:989-1010 (bernoulli mask / keep_prob, identity when
// p == 0 or in eval mode).
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace ntb {

__device__ __forceinline__ uint4 philox4x32_10(uint4 ctr, uint2 key) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      key.x += W0;
      key.y += W1;
    }
    const uint32_t lo0 = M0 * ctr.x, hi0 = __umulhi(M0, ctr.x);
    const uint32_t lo1 = M1 * ctr.z, hi1 = __umulhi(M1, ctr.z);
    ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
  }
  return ctr;
}

template <typename T>
__device__ __forceinline__ float ld1(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld1<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld1<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ void st1(T* p, int64_t i, float v);
template <>
__device__ __forceinline__ void st1<float>(float* p, int64_t i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void st1<__nv_bfloat16>(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16(v);
}

// One thread per group of 4 elements (one Philox block); grid-stride.
template <typename T>
__global__ void dropout_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n, float p, float scale,
                               uint64_t seed) {
  const uint2 key = make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  const int64_t groups = (n + 3) / 4;
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 r = philox4x32_10(make_uint4(static_cast<uint32_t>(g), static_cast<uint32_t>(g >> 32), 0u, 0u), key);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
    const int64_t base = g * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t i = base + j;
      if (i < n) {
        const float u = static_cast<float>(w[j] >> 8) * (1.0f / 16777216.0f);
        st1(y, i, u >= p ? ld1(x, i) * scale : 0.f);
      }
    }
  }
}

// y = dropout(x) with the mask of (seed); x contiguous bf16 or fp32.
at::Tensor dropout_apply(const at::Tensor& x, double p, int64_t seed) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous(), "dropout: contiguous CUDA tensor");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat, "dropout: bf16 or fp32");
  TORCH_CHECK(p >= 0.0 && p < 1.0, "dropout: p in [0, 1)");
  at::Tensor y = at::empty_like(x);
  const int64_t n = x.numel();
  if (n == 0) return y;
  const int dev = x.get_device();
  const int64_t groups = (n + 3) / 4;
  const int blocks = static_cast<int>(std::min<int64_t>((groups + 255) / 256, 8L * num_sms(dev)));
  const float scale = static_cast<float>(1.0 / (1.0 - p));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  if (x.scalar_type() == at::kBFloat16)
    dropout_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                               reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), n,
                                               static_cast<float>(p), scale, static_cast<uint64_t>(seed));
  else
    dropout_kernel<<<blocks, 256, 0, stream>>>(x.data_ptr<float>(), y.data_ptr<float>(), n, static_cast<float>(p),
                                               scale, static_cast<uint64_t>(seed));
  NTB_LAUNCH_CHECK(1);
  return y;
}

}  // namespace ntb
