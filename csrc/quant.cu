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

// Eight consecutive elements <-> floats (16-byte bf16 or 2 x 16-byte fp32 accesses).
__device__ __forceinline__ void load8(const bf16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
  v[4] = bf16_lo(u.z); v[5] = bf16_hi(u.z); v[6] = bf16_lo(u.w); v[7] = bf16_hi(u.w);
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8(bf16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                            pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Quantises 8 values with scale s (the correctly rounded quotient, as the recipe states
// q = e4m3(x / s); div_scale), optionally stochastically; returns the 8 codes packed little-endian,
// and with DQ the dequantised values.
template <bool DQ = true>
__device__ __forceinline__ uint2 quant8(const float (&v)[8], float s, bool stochastic, uint64_t seed, int64_t idx0,
                                        float (&dq)[8]) {
  const ScaleDiv sd = make_scale_div(s);
  float y[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    y[j] = div_scale(v[j], sd);
    // nearest: the saturating conversion clamps to +-448 itself; stochastic rounding needs |y| <= 448
    if (stochastic)
      y[j] = e4m3_sr(fminf(fmaxf(y[j], -448.f), 448.f), uniform01(seed, static_cast<uint64_t>(idx0 + j)));
  }
  uint32_t w[2];
#pragma unroll
  for (int h = 0; h < 2; ++h)
    w[h] = to_e4m3x2(y[4 * h], y[4 * h + 1]) | (to_e4m3x2(y[4 * h + 2], y[4 * h + 3]) << 16);
  if (DQ) {
#pragma unroll
    for (int j = 0; j < 8; ++j) dq[j] = from_e4m3(static_cast<uint8_t>(w[j >> 2] >> (8 * (j & 3)))) * s;
  }
  return make_uint2(w[0], w[1]);
}

// 1x128 tiles: a half-warp per (row, 128-column tile), 8 elements (one 16-byte load) per lane; the
// tile's amax is reduced over the 16 lanes with shuffles. Writes the codes (8-byte stores), the
// scale, and optionally the dequantised value. Grid-stride over tile pairs.
template <typename T, bool DQ>
__global__ void __launch_bounds__(256) quant_tile_kernel(const T* __restrict__ x, int64_t rows, int cols,
                                                         uint8_t* __restrict__ q, float* __restrict__ scales,
                                                         T* __restrict__ dq, int stochastic, uint64_t seed) {
  // Tile t (1 x 128) of the contiguous [rows, cols] matrix covers elements [128 t, 128 t + 128) and
  // owns scale t. A warp holds two tiles (one per half warp) and keeps two such pairs in flight per
  // iteration, so each thread has 32 bytes of loads outstanding before it reduces.
  const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
  const int64_t tiles = rows * (cols / 128);
  const int64_t pairs = (tiles + 1) / 2;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w < pairs;
       w += 2 * nwarps) {
    int64_t t[2];
    bool live[2];
    float v[2][8];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      t[u] = 2 * (w + u * nwarps) + half;
      live[u] = t[u] < tiles;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[u][j] = 0.f;
      if (live[u]) load8(x + t[u] * 128 + hl * 8, v[u]);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[u][j]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (!live[u]) continue;
      const float s = amax > 0.f ? amax / 448.f : 1.f;
      if (hl == 0) scales[t[u]] = s;
      const int64_t idx0 = t[u] * 128 + hl * 8;
      float d[8];
      const uint2 codes = quant8<DQ>(v[u], s, stochastic != 0, seed, idx0, d);
      if (q) *reinterpret_cast<uint2*>(q + idx0) = codes;
      if (DQ) store8(dq + idx0, d);
    }
  }
}

// 128x128 blocks: one CTA (256 threads) per block; pass 1 reduces the block's amax from 16-byte
// loads (each thread 8 rows x 8 columns), pass 2 re-reads the block (L2-resident) and quantises.
// The source may be a stack of groups read in place: row r lives at (r / rpg) * gstride + (r % rpg) *
// cols (rpg = rows and gstride = 0 for a plain matrix; rpg a multiple of 128 otherwise, so no block
// spans two groups). Codes, scales and dequantised values are written as one contiguous matrix.
template <typename T>
__global__ void __launch_bounds__(256) quant_block_kernel(const T* __restrict__ x, int64_t rows, int cols,
                                                          uint8_t* __restrict__ q, float* __restrict__ scales,
                                                          T* __restrict__ dq, int stochastic, uint64_t seed,
                                                          int64_t rpg, int64_t gstride) {
  __shared__ float red[8];
  const int nbc = cols / 128;
  const int64_t br = blockIdx.x / nbc;
  const int bc = blockIdx.x % nbc;
  const int64_t r0 = br * 128;
  const int c8 = (threadIdx.x & 15) * 8;  // column chunk of this thread
  const int rsub = threadIdx.x >> 4;      // rows rsub, rsub + 16, ...
  const T* xb = x + (r0 / rpg) * gstride - (r0 / rpg) * rpg * cols;  // row r of this block at xb + r * cols
  float amax = 0.f;
  for (int i = 0; i < 8; ++i) {
    const int64_t r = r0 + rsub + 16 * i;
    if (r >= rows) break;
    float v[8];
    load8(xb + r * cols + bc * 128 + c8, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
  }
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float a = red[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) a = fmaxf(a, red[k]);
  const float s = a > 0.f ? a / 448.f : 1.f;
  if (threadIdx.x == 0) scales[br * nbc + bc] = s;
  for (int i = 0; i < 8; ++i) {
    const int64_t r = r0 + rsub + 16 * i;
    if (r >= rows) break;
    const int64_t idx0 = r * cols + bc * 128 + c8;
    float v[8], d[8];
    load8(xb + idx0, v);
    const uint2 codes = quant8(v, s, stochastic != 0, seed, idx0, d);
    if (q) *reinterpret_cast<uint2*>(q + idx0) = codes;
    if (dq) store8(dq + idx0, d);
  }
}

// Dequantise e4m3 bytes with tile (block_rows = 1) or block (128) scales, 8 codes per thread.
template <typename T>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scales,
                                                      int64_t rows, int cols, int block_rows, T* __restrict__ out) {
  const int64_t n8 = rows * cols / 8;
  const int ntc = cols / 128;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t r = e / cols;
    const int c = static_cast<int>(e - r * cols);
    const float s = scales[(r / block_rows) * ntc + c / 128];
    const uint2 u = *reinterpret_cast<const uint2*>(q + e);
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = from_e4m3(static_cast<uint8_t>(u.x >> (8 * j))) * s;
      v[4 + j] = from_e4m3(static_cast<uint8_t>(u.y >> (8 * j))) * s;
    }
    store8(out + e, v);
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
      const int64_t pairs = (rows * (cols / 128) + 1) / 2;
      const int grid = static_cast<int>(std::min<int64_t>((pairs + 7) / 8, 16L * num_sms(x.get_device())));
      if (dq)
        quant_tile_kernel<bf16, true><<<grid, 256, 0, stream>>>(xp, rows, cols, q, s, reinterpret_cast<bf16*>(dq),
                                                                stochastic, sd);
      else
        quant_tile_kernel<bf16, false><<<grid, 256, 0, stream>>>(xp, rows, cols, q, s, nullptr, stochastic, sd);
    } else {
      const int64_t blocks = ((rows + 127) / 128) * (cols / 128);
      quant_block_kernel<bf16><<<blocks, 256, 0, stream>>>(xp, rows, cols, q, s, reinterpret_cast<bf16*>(dq),
                                                           stochastic, sd, rows, 0);
    }
  } else {
    TORCH_CHECK(x.scalar_type() == at::kFloat, "fp8 quantiser: bf16 or fp32 input");
    const float* xp = x.data_ptr<float>();
    if (block_rows == 1) {
      const int64_t pairs = (rows * (cols / 128) + 1) / 2;
      const int grid = static_cast<int>(std::min<int64_t>((pairs + 7) / 8, 16L * num_sms(x.get_device())));
      if (dq)
        quant_tile_kernel<float, true><<<grid, 256, 0, stream>>>(xp, rows, cols, q, s, reinterpret_cast<float*>(dq),
                                                                 stochastic, sd);
      else
        quant_tile_kernel<float, false><<<grid, 256, 0, stream>>>(xp, rows, cols, q, s, nullptr, stochastic, sd);
    } else {
      const int64_t blocks = ((rows + 127) / 128) * (cols / 128);
      quant_block_kernel<float><<<blocks, 256, 0, stream>>>(xp, rows, cols, q, s, reinterpret_cast<float*>(dq),
                                                            stochastic, sd, rows, 0);
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

// Rounds a stack of `groups` matrices [rows_per_group, cols] (bf16), read in place from `src` at
// element offsets g * group_stride, through e4m3 with 128 x 128 block scales; returns the rounded
// stack as one contiguous [groups * rows_per_group, cols] matrix. `src` only supplies the start
// address (its storage must hold every group).
at::Tensor fp8_quant_dequant_strided(const at::Tensor& src, int64_t groups, int64_t rows_per_group, int64_t cols,
                                     int64_t group_stride) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16, "fp8_quant_dequant_strided: bf16 CUDA source");
  TORCH_CHECK(groups >= 1 && rows_per_group % 128 == 0 && cols % 128 == 0 && group_stride >= rows_per_group * cols &&
                  group_stride % 8 == 0,
              "fp8_quant_dequant_strided: rows per group and columns must be multiples of 128, groups must not overlap");
  const int64_t need = (src.storage_offset() + (groups - 1) * group_stride + rows_per_group * cols) * 2;
  TORCH_CHECK(static_cast<int64_t>(src.storage().nbytes()) >= need && (reinterpret_cast<uintptr_t>(src.data_ptr()) & 15) == 0,
              "fp8_quant_dequant_strided: source storage too small or misaligned");
  const int64_t rows = groups * rows_per_group;
  auto out = at::empty({rows, cols}, src.options());
  auto s = at::empty({rows / 128, cols / 128}, src.options().dtype(at::kFloat));
  const int64_t blocks = (rows / 128) * (cols / 128);
  quant_block_kernel<bf16><<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(src.data_ptr()), rows, static_cast<int>(cols), nullptr, s.data_ptr<float>(),
      reinterpret_cast<bf16*>(out.data_ptr()), 0, 0, rows_per_group, group_stride);
  NTB_LAUNCH_CHECK(1);
  return out;
}

// Same reading of a strided stack, returning the e4m3 codes [groups * rows_per_group, cols] and the
// 128 x 128 block scales [groups * rows_per_group / 128, cols / 128] (the B operand of the grouped
// fp8 GEMM).
std::vector<at::Tensor> fp8_quantize_strided(const at::Tensor& src, int64_t groups, int64_t rows_per_group,
                                             int64_t cols, int64_t group_stride) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16, "fp8_quantize_strided: bf16 CUDA source");
  TORCH_CHECK(groups >= 1 && rows_per_group % 128 == 0 && cols % 128 == 0 && group_stride >= rows_per_group * cols &&
                  group_stride % 8 == 0,
              "fp8_quantize_strided: rows per group and columns must be multiples of 128, groups must not overlap");
  const int64_t need = (src.storage_offset() + (groups - 1) * group_stride + rows_per_group * cols) * 2;
  TORCH_CHECK(static_cast<int64_t>(src.storage().nbytes()) >= need && (reinterpret_cast<uintptr_t>(src.data_ptr()) & 15) == 0,
              "fp8_quantize_strided: source storage too small or misaligned");
  const int64_t rows = groups * rows_per_group;
  auto q = at::empty({rows, cols}, src.options().dtype(at::kByte));
  auto s = at::empty({rows / 128, cols / 128}, src.options().dtype(at::kFloat));
  const int64_t blocks = (rows / 128) * (cols / 128);
  quant_block_kernel<bf16><<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(src.data_ptr()), rows, static_cast<int>(cols), q.data_ptr<uint8_t>(),
      s.data_ptr<float>(), nullptr, 0, 0, rows_per_group, group_stride);
  NTB_LAUNCH_CHECK(1);
  return {q, s};
}

// Codes and scales of a 1x128-tile quantisation plus the dequantised (rounded) values, in one pass.
std::vector<at::Tensor> fp8_quantize_with_dq(const at::Tensor& x, bool stochastic, int64_t seed) {
  check_quant_input(x, 1);
  const int64_t rows = x.size(0), cols = x.size(1);
  auto q = at::empty({rows, cols}, x.options().dtype(at::kByte));
  auto s = at::empty({rows, cols / 128}, x.options().dtype(at::kFloat));
  auto dq = at::empty_like(x);
  if (rows == 0) return {q, s, dq};
  launch_quant(x, 1, stochastic, seed, q.data_ptr<uint8_t>(), s.data_ptr<float>(), dq.data_ptr());
  return {q, s, dq};
}

at::Tensor fp8_dequantize(const at::Tensor& q, const at::Tensor& scales, int64_t block_rows, at::ScalarType dtype) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 2 && q.is_contiguous() && q.scalar_type() == at::kByte, "fp8_dequantize: q");
  const int64_t rows = q.size(0);
  const int cols = static_cast<int>(q.size(1));
  auto out = at::empty({rows, cols}, q.options().dtype(dtype));
  if (rows == 0) return out;
  TORCH_CHECK(cols % 128 == 0, "fp8_dequantize: columns must be a multiple of 128");
  auto stream = at::cuda::getCurrentCUDAStream();
  const int64_t n8 = rows * cols / 8;
  const int blocks = static_cast<int>(std::min<int64_t>((n8 + 255) / 256, 16L * num_sms(q.get_device())));
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
