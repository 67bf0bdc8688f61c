// fp8 (e4m3) quantisers of the DeepSeek-V3 recipe for sm_100a.
//
//   tile_1x128    : one fp32 scale per (row, 128-column tile)     - activations
//   block_128x128 : one fp32 scale per 128 x 128 block            - weights
//
// scale = amax / 448 (1 if the tile is all zero), q = e4m3(x / scale) with
// round-to-nearest-even (CUDA's satfinite conversion) or stochastic rounding:
// y is written as down + frac * ulp with ulp the e4m3 spacing at |y| (2^(e-3)
// for normal values, 2^-9 below 2^-6), and rounds up with probability frac.
// Random bits come from the "lowbias32" integer hash (C. Wellons, public
// domain) of (seed, element index), so a kernel is deterministic per seed.
//
// Reference parity: src/runtime/te_backend.py:61-204 emulates this on an int8
// grid in fp32; src/models/moe.py:72-143 does the same for MoE payloads.
#include <ATen/cuda/CUDAContext.h>
#include <cuda_fp8.h>
#include <torch/extension.h>

#include "common.cuh"
#include "fp8_util.cuh"
#include "host_utils.h"

namespace ntb {

using bf16 = __nv_bfloat16;

template <typename T>
__device__ __forceinline__ float ldf(const T* p);
template <>
__device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldf<bf16>(const bf16* p) { return __bfloat162float(*p); }

template <typename T>
__device__ __forceinline__ void stf(T* p, float v);
template <>
__device__ __forceinline__ void stf<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void stf<bf16>(bf16* p, float v) { *p = __float2bfloat16(v); }

// One warp per (row, 128-column tile). Writes q (optional), scale, and the
// dequantised value (optional).
template <typename T>
__global__ void quant_tile_kernel(const T* __restrict__ x, int64_t rows, int cols, uint8_t* __restrict__ q,
                                  float* __restrict__ scales, T* __restrict__ dq, int stochastic, uint64_t seed) {
  const int warps = blockDim.x >> 5;
  const int64_t tile = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int ntc = cols / 128;
  if (tile >= rows * ntc) return;
  const int64_t r = tile / ntc;
  const int tc = tile % ntc;
  const int64_t base = r * cols + tc * 128;
  float v[4];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = ldf(x + base + lane * 4 + j);
    amax = fmaxf(amax, fabsf(v[j]));
  }
  amax = warp_max(amax);
  const float s = amax > 0.f ? amax / 448.f : 1.f;
  if (lane == 0) scales[r * ntc + tc] = s;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t idx = base + lane * 4 + j;
    float y = fminf(fmaxf(v[j] / s, -448.f), 448.f);
    if (stochastic) y = e4m3_sr(y, uniform01(seed, static_cast<uint64_t>(idx)));
    const uint8_t b = to_e4m3(y);
    if (q) q[idx] = b;
    if (dq) stf(dq + idx, from_e4m3(b) * s);
  }
}

// One CTA (256 threads) per 128 x 128 block.
template <typename T>
__global__ void quant_block_kernel(const T* __restrict__ x, int64_t rows, int cols, uint8_t* __restrict__ q,
                                   float* __restrict__ scales, T* __restrict__ dq, int stochastic, uint64_t seed) {
  __shared__ float red[8];
  const int nbc = cols / 128;
  const int64_t br = blockIdx.x / nbc;
  const int bc = blockIdx.x % nbc;
  const int64_t r0 = br * 128;
  float amax = 0.f;
  for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) {
    const int64_t r = r0 + i / 128;
    if (r < rows) amax = fmaxf(amax, fabsf(ldf(x + r * cols + bc * 128 + (i % 128))));
  }
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float a = red[0];
  const float s = a > 0.f ? a / 448.f : 1.f;
  if (threadIdx.x == 0) scales[br * nbc + bc] = s;
  for (int i = threadIdx.x; i < 128 * 128; i += blockDim.x) {
    const int64_t r = r0 + i / 128;
    if (r >= rows) continue;
    const int64_t idx = r * cols + bc * 128 + (i % 128);
    float y = fminf(fmaxf(ldf(x + idx) / s, -448.f), 448.f);
    if (stochastic) y = e4m3_sr(y, uniform01(seed, static_cast<uint64_t>(idx)));
    const uint8_t b = to_e4m3(y);
    if (q) q[idx] = b;
    if (dq) stf(dq + idx, from_e4m3(b) * s);
  }
}

// Dequantise e4m3 bytes with tile (block_rows = 1) or block (128) scales.
template <typename T>
__global__ void dequant_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scales, int64_t rows, int cols,
                               int block_rows, T* __restrict__ out) {
  const int64_t n = rows * cols;
  const int ntc = cols / 128;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols;
    const int c = i % cols;
    const float s = scales[(r / block_rows) * ntc + c / 128];
    stf(out + i, from_e4m3(q[i]) * s);
  }
}

static void launch_quant(const at::Tensor& x, int block_rows, bool stochastic, int64_t seed, uint8_t* q, float* s,
                         void* dq) {
  const int64_t rows = x.size(0);
  const int cols = static_cast<int>(x.size(1));
  auto stream = at::cuda::getCurrentCUDAStream();
  const uint64_t sd = static_cast<uint64_t>(seed);
  if (x.scalar_type() == at::kBFloat16) {
    const bf16* xp = reinterpret_cast<const bf16*>(x.data_ptr());
    if (block_rows == 1) {
      const int64_t tiles = rows * (cols / 128);
      quant_tile_kernel<bf16><<<(tiles + 7) / 8, 256, 0, stream>>>(xp, rows, cols, q, s, reinterpret_cast<bf16*>(dq),
                                                                  stochastic, sd);
    } else {
      const int64_t blocks = ((rows + 127) / 128) * (cols / 128);
      quant_block_kernel<bf16><<<blocks, 256, 0, stream>>>(xp, rows, cols, q, s, reinterpret_cast<bf16*>(dq),
                                                           stochastic, sd);
    }
  } else {
    TORCH_CHECK(x.scalar_type() == at::kFloat, "fp8 quantiser: bf16 or fp32 input");
    const float* xp = x.data_ptr<float>();
    if (block_rows == 1) {
      const int64_t tiles = rows * (cols / 128);
      quant_tile_kernel<float><<<(tiles + 7) / 8, 256, 0, stream>>>(xp, rows, cols, q, s, reinterpret_cast<float*>(dq),
                                                                   stochastic, sd);
    } else {
      const int64_t blocks = ((rows + 127) / 128) * (cols / 128);
      quant_block_kernel<float><<<blocks, 256, 0, stream>>>(xp, rows, cols, q, s, reinterpret_cast<float*>(dq),
                                                            stochastic, sd);
    }
  }
  NTB_LAUNCH_CHECK(1);
}

static void check_quant_input(const at::Tensor& x, int64_t block_rows) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "fp8 quantiser: contiguous 2-D CUDA tensor");
  TORCH_CHECK(x.size(1) % 128 == 0, "fp8 quantiser: columns must be a multiple of 128");
  TORCH_CHECK(block_rows == 1 || block_rows == 128, "fp8 quantiser: block_rows must be 1 or 128");
}

// Returns (q uint8 [R, C], scales fp32 [ceil(R / block_rows), C / 128]).
std::vector<at::Tensor> fp8_quantize(const at::Tensor& x, int64_t block_rows, bool stochastic, int64_t seed) {
  check_quant_input(x, block_rows);
  const int64_t rows = x.size(0), cols = x.size(1);
  auto q = at::empty({rows, cols}, x.options().dtype(at::kByte));
  auto s = at::empty({(rows + block_rows - 1) / block_rows, cols / 128}, x.options().dtype(at::kFloat));
  if (rows == 0) return {q, s};
  launch_quant(x, static_cast<int>(block_rows), stochastic, seed, q.data_ptr<uint8_t>(), s.data_ptr<float>(), nullptr);
  return {q, s};
}

at::Tensor fp8_quant_dequant(const at::Tensor& x, int64_t block_rows, bool stochastic, int64_t seed) {
  check_quant_input(x, block_rows);
  const int64_t rows = x.size(0), cols = x.size(1);
  auto out = at::empty_like(x);
  auto s = at::empty({(rows + block_rows - 1) / block_rows, cols / 128}, x.options().dtype(at::kFloat));
  if (rows == 0) return out;
  launch_quant(x, static_cast<int>(block_rows), stochastic, seed, nullptr, s.data_ptr<float>(), out.data_ptr());
  return out;
}

at::Tensor fp8_dequantize(const at::Tensor& q, const at::Tensor& scales, int64_t block_rows, at::ScalarType dtype) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 2 && q.is_contiguous() && q.scalar_type() == at::kByte, "fp8_dequantize: q");
  const int64_t rows = q.size(0);
  const int cols = static_cast<int>(q.size(1));
  auto out = at::empty({rows, cols}, q.options().dtype(dtype));
  if (rows == 0) return out;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int64_t n = rows * cols;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 16));
  if (dtype == at::kBFloat16)
    dequant_kernel<bf16><<<blocks, 256, 0, stream>>>(q.data_ptr<uint8_t>(), scales.data_ptr<float>(), rows, cols,
                                                     static_cast<int>(block_rows), reinterpret_cast<bf16*>(out.data_ptr()));
  else
    dequant_kernel<float><<<blocks, 256, 0, stream>>>(q.data_ptr<uint8_t>(), scales.data_ptr<float>(), rows, cols,
                                                      static_cast<int>(block_rows), out.data_ptr<float>());
  NTB_LAUNCH_CHECK(1);
  return out;
}

}  // namespace ntb
