// Persistent low-bit weight copies for sm_100a: the refresh that runs once per optimizer
// step (amax per output channel or per tensor, then e4m3 codes or NF4 codes packed two per
// byte) and the dequantisation the straight-through forward reads.
//
//   fp8:  scale = amax / 448 (1 if zero), q = e4m3(clamp(w / scale, +-448)) (round to nearest even)
//   nf4:  scale = amax (1 if zero), code = index of the nearest of the 16 NF4 levels to w / scale
//         (the first one on a tie), element i of the flattened weight in byte i / 2, low nibble
//         first
// One launch computes the scales (a block per row, or a grid-wide max for per-tensor scales),
// a second writes the codes; the arithmetic is the same fp32 sequence as the PyTorch
// statement of the format, so both give the same bits.
//
// Reference parity: src/layers.py:60-184 (NF4 codebook, packing, quantisers) and 353-436
// (refresh of the persistent buffers after each optimizer step).
#include <ATen/cuda/CUDAContext.h>
#include <cuda_fp8.h>
#include <torch/extension.h>

#include "common.cuh"
#include "fp8_util.cuh"
#include "host_utils.h"

namespace ntb {

__constant__ float kNf4Levels[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f, -0.28444138169288635f,
    -0.18477343022823334f, -0.09105003625154495f, 0.0f, 0.07958029955625534f, 0.16093020141124725f,
    0.24611230194568634f, 0.33791524171829224f, 0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f,
    1.0f};

template <typename T>
__device__ __forceinline__ float pld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float pld<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float pld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

// amax of each row (per_channel) into amax[row]; per_tensor: every block folds its part into
// amax[0] (zeroed by the host) with an atomic max on the float bits.
template <typename T>
__global__ void persistent_amax_kernel(const T* __restrict__ w, int64_t rows, int64_t cols, bool per_tensor,
                                       float* __restrict__ amax) {
  __shared__ float part[32];
  float m = 0.f;
  if (per_tensor) {
    const int64_t n = rows * cols;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
      m = fmaxf(m, fabsf(pld(w, i)));
  } else {
    const int64_t r = blockIdx.x;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, fabsf(pld(w, r * cols + c)));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    m = warp_max(m);
    if (threadIdx.x == 0) {
      if (per_tensor)
        atomicMax(reinterpret_cast<unsigned int*>(amax), __float_as_uint(m));
      else
        amax[blockIdx.x] = m;
    }
  }
}

// amax -> scale in place.
__global__ void persistent_scale_kernel(float* __restrict__ s, int64_t n, float qmax) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) {
    const float v = s[i] / qmax;
    s[i] = v > 0.f ? v : 1.f;
  }
}

// One thread per pair of flattened elements (2p, 2p + 1).
template <typename T>
__global__ void persistent_quant_kernel(const T* __restrict__ w, int64_t numel, int64_t cols, bool per_tensor,
                                        bool nf4, const float* __restrict__ scale, uint8_t* __restrict__ out) {
  const int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t i0 = 2 * p;
  if (i0 >= numel) return;
  uint32_t code[2] = {0u, 0u};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int64_t i = i0 + h;
    if (i >= numel) break;
    const float s = per_tensor ? scale[0] : scale[i / cols];
    const float y = pld(w, i) / s;
    if (nf4) {
      int best = 0;
      float bd = fabsf(y - kNf4Levels[0]);
#pragma unroll
      for (int l = 1; l < 16; ++l) {
        const float d = fabsf(y - kNf4Levels[l]);
        if (d < bd) {
          bd = d;
          best = l;
        }
      }
      code[h] = static_cast<uint32_t>(best);
    } else {
      out[i] = to_e4m3(fminf(fmaxf(y, -448.f), 448.f));
    }
  }
  if (nf4) out[p] = static_cast<uint8_t>(code[0] | (code[1] << 4));
}

template <typename T>
__global__ void persistent_dequant_kernel(const uint8_t* __restrict__ q, int64_t numel, int64_t cols, bool per_tensor,
                                          bool nf4, const float* __restrict__ scale, T* __restrict__ out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= numel) return;
  const float s = per_tensor ? scale[0] : scale[i / cols];
  const float v = nf4 ? kNf4Levels[(q[i >> 1] >> (4 * (i & 1))) & 0xF] : from_e4m3(q[i]);
  if constexpr (std::is_same<T, float>::value)
    out[i] = v * s;
  else
    out[i] = __float2bfloat16(v * s);
}

// {codes, scale}: fp8 codes [rows, cols] (uint8 bits of e4m3) or NF4 bytes [ceil(numel / 2)];
// scale [rows] (per channel) or [1].
std::vector<at::Tensor> persistent_quantize(const at::Tensor& w, bool nf4, bool per_tensor) {
  TORCH_CHECK(w.is_cuda() && w.dim() == 2 && w.is_contiguous(), "persistent_quantize: 2-D contiguous CUDA weight");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 || w.scalar_type() == at::kFloat, "persistent_quantize: bf16 or fp32");
  const int64_t rows = w.size(0), cols = w.size(1), numel = rows * cols;
  const int dev = w.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  auto f32 = w.options().dtype(at::kFloat);
  at::Tensor scale = per_tensor ? at::zeros({1}, f32) : at::empty({rows}, f32);
  at::Tensor codes = nf4 ? at::empty({(numel + 1) / 2}, w.options().dtype(at::kByte))
                         : at::empty({rows, cols}, w.options().dtype(at::kByte));
  if (numel == 0) {
    if (per_tensor) scale.fill_(1.f);
    return {codes, scale};
  }
  const bool bf = w.scalar_type() == at::kBFloat16;
  const int amax_blocks = per_tensor ? static_cast<int>(std::min<int64_t>((numel + 255) / 256, 4L * num_sms(dev)))
                                     : static_cast<int>(rows);
  if (bf)
    persistent_amax_kernel<<<amax_blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                                                            rows, cols, per_tensor, scale.data_ptr<float>());
  else
    persistent_amax_kernel<<<amax_blocks, 256, 0, stream>>>(w.data_ptr<float>(), rows, cols, per_tensor,
                                                            scale.data_ptr<float>());
  const int64_t ns = scale.numel();
  persistent_scale_kernel<<<static_cast<int>((ns + 255) / 256), 256, 0, stream>>>(scale.data_ptr<float>(), ns,
                                                                                  nf4 ? 1.f : 448.f);
  const int qblocks = static_cast<int>(((numel + 1) / 2 + 255) / 256);
  if (bf)
    persistent_quant_kernel<<<qblocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), numel,
                                                         cols, per_tensor, nf4, scale.data_ptr<float>(),
                                                         codes.data_ptr<uint8_t>());
  else
    persistent_quant_kernel<<<qblocks, 256, 0, stream>>>(w.data_ptr<float>(), numel, cols, per_tensor, nf4,
                                                         scale.data_ptr<float>(), codes.data_ptr<uint8_t>());
  NTB_LAUNCH_CHECK(3);
  return {codes, scale};
}

at::Tensor persistent_dequantize(const at::Tensor& codes, const at::Tensor& scale, int64_t rows, int64_t cols,
                                 bool nf4, at::ScalarType dtype) {
  TORCH_CHECK(codes.is_cuda() && codes.scalar_type() == at::kByte && codes.is_contiguous(),
              "persistent_dequantize: uint8 CUDA codes");
  const int64_t numel = rows * cols;
  TORCH_CHECK(codes.numel() == (nf4 ? (numel + 1) / 2 : numel), "persistent_dequantize: code count");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && (scale.numel() == 1 || scale.numel() == rows),
              "persistent_dequantize: fp32 scale [rows] or [1]");
  TORCH_CHECK(dtype == at::kBFloat16 || dtype == at::kFloat, "persistent_dequantize: bf16 or fp32 output");
  at::Tensor out = at::empty({rows, cols}, codes.options().dtype(dtype));
  if (numel == 0) return out;
  const bool per_tensor = scale.numel() == 1;  // with one row the two granularities coincide
  const int dev = codes.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  const int blocks = static_cast<int>((numel + 255) / 256);
  if (dtype == at::kBFloat16)
    persistent_dequant_kernel<<<blocks, 256, 0, stream>>>(codes.data_ptr<uint8_t>(), numel, cols, per_tensor, nf4,
                                                          scale.data_ptr<float>(),
                                                          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  else
    persistent_dequant_kernel<<<blocks, 256, 0, stream>>>(codes.data_ptr<uint8_t>(), numel, cols, per_tensor, nf4,
                                                          scale.data_ptr<float>(), out.data_ptr<float>());
  NTB_LAUNCH_CHECK(1);
  return out;
}

}  // namespace ntb
