// NVFP4 on the 5th-generation tensor cores (sm_100a): quantiser, dequantiser and a
// block-scaled GEMM that runs tcgen05.mma kind::mxf4nvf4 with the scale factors applied
// by the tensor core itself.
//
// Format (one matrix [R, K], K a multiple of 64):
//   q   uint8 [R, K/2]  e2m1 values, element k of a row in byte k/2 (low nibble for even k)
//   sf  uint8 e4m3 block scales, one per 1 x 16 group, stored in the tensor core's
//       scale-factor blocks: 128 rows x 4 scales (64 columns of the matrix) = 512 bytes;
//       block (rb, kb) at byte (rb * K/64 + kb) * 512, and inside a block the scale of
//       row r, group j at (r % 32) * 16 + ((r % 128) / 32) * 4 + (j % 4). Rows past R in the
//       last row block hold 0. Size: ceil(R/128) * (K/64) * 512 bytes.
//   gs  fp32 [1] per-tensor scale: x ~= e2m1 * e4m3 * gs with gs = amax / (6 * 448).
// This is the NVFP4 recipe of the GPT-1.3B fp4 configuration (e2m1 in 1x16 blocks with e4m3
// scales); the reference only emulates low-bit GEMMs in fp32 (src/runtime/te_backend.py:
// 229-260 with the fp4 mode of src/runtime/mixed_precision.py:635-762).
//
// GEMM: C[M, N] (bf16) = gs_a * gs_b * sum_k (qa * sfa)[m, k] (qb * sfb)[n, k] (+ bias), both
// operands K-major, K a multiple of 256. Persistent CTAs, one per SM, 320 threads, 128 x 256
// output tiles, 256-element (128-byte) K tiles in a 4-stage ring:
//   warp 0      producer: per K tile one TMA box of A (128 rows x 128 B) and two of B, plus
//               plain bulk copies of the tile's scale blocks (A: 4 x 512 B; B: 2 x 4 x 512 B),
//               all on one mbarrier (no cluster multicast: this GEMM may run inside a
//               multi-GPU job)
//   warp 1      allocates TMEM; one thread copies the scale blocks of the K tile from shared
//               memory into TMEM (tcgen05.cp 32x128b.warpx4: 4 columns per 128 rows, the same
//               bytes in every lane quarter) and issues 4 x tcgen05.mma kind::mxf4nvf4
//               block16 (128 x 256 x 64) into the fp32 accumulator. The copy and the MMAs of a
//               thread execute in issue order, so one scale region is reused every K tile.
//   warps 2..9  epilogue: two warps per TMEM lane quarter, 128 columns each; they load the
//               accumulator into registers, release it (the next tile's MMAs start while
//               they scale, add the bias and store bf16).
// TMEM: accumulator columns [0, 256), A scales [256, 272), B scales [272, 304).
// Every wait is bounded (common.cuh) and reports through the device status word.
#include <ATen/cuda/CUDAContext.h>
#include <cuda_fp8.h>
#include <torch/extension.h>

#include "common.cuh"
#include "fp8_util.cuh"
#include "host_utils.h"

namespace ntb {

namespace fp4g {
constexpr int BM = 128, BN = 256;
constexpr int BK = 256;                 // elements per K tile
constexpr int BKB = BK / 2;             // bytes per row per K tile (= one 128-byte swizzle row)
constexpr int KK = BK / 64;             // MMAs (K = 64) per K tile
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BKB;       // 16 KB
constexpr int B_BYTES = BN * BKB;       // 32 KB
constexpr int SFA_BYTES = KK * 512;     // 2 KB: one 512-byte block per MMA
constexpr int SFB_BYTES = 2 * KK * 512; // 4 KB: two 128-row halves
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
constexpr int THREADS = 320;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t SFA_COL = 256, SFB_COL = 272;
}  // namespace fp4g

// ---------------------------------------------------------------- device helpers
// Eight fp32 values -> eight e2m1 nibbles (round to nearest even, saturating), element 0
// in the low nibble of byte 0.
__device__ __forceinline__ uint32_t pack_e2m1x8(const float (&v)[8]) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}\n"
      : "=r"(out)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return out;
}

// e2m1 code (sign bit 3, exponent bits 2..1, mantissa bit 0) -> value.
__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const uint32_t m = c & 7u;
  const float mag = m < 2u ? 0.5f * static_cast<float>(m)
                           : ldexpf(1.f + 0.5f * static_cast<float>(m & 1u), static_cast<int>(m >> 1) - 1);
  return (c & 8u) ? -mag : mag;
}

__device__ __forceinline__ int64_t sf_offset(int64_t r, int64_t j, int64_t kblocks) {
  return ((r >> 7) * kblocks + (j >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (j & 3);
}

__device__ __forceinline__ float gscale_of(float amax) {
  const float g = amax / 2688.f;  // 6 (largest e2m1) * 448 (largest e4m3)
  return g > 0.f ? g : 1.f;
}

template <typename T>
__device__ __forceinline__ void load16(const T* p, float (&v)[16]);
template <>
__device__ __forceinline__ void load16<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[16]) {
  const uint4* s = reinterpret_cast<const uint4*>(p);
  const uint4 a = __ldg(s), b = __ldg(s + 1);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = bf16_lo(w[i]);
    v[2 * i + 1] = bf16_hi(w[i]);
  }
}
template <>
__device__ __forceinline__ void load16<float>(const float* p, float (&v)[16]) {
  const float4* s = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 t = __ldg(s + i);
    v[4 * i] = t.x;
    v[4 * i + 1] = t.y;
    v[4 * i + 2] = t.z;
    v[4 * i + 3] = t.w;
  }
}

// ---------------------------------------------------------------- quantiser
// |x| max over the tensor into amax (zeroed by the host), as float bits (non-negative floats
// order like their bit patterns).
template <typename T>
__global__ void nvfp4_amax_kernel(const T* __restrict__ x, int64_t n16, float* __restrict__ amax) {
  float m = 0.f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v[16];
    load16(x + i * 16, v);
#pragma unroll
    for (int t = 0; t < 16; ++t) m = fmaxf(m, fabsf(v[t]));
  }
  m = warp_max(m);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    m = warp_max(m);
    if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned int*>(amax), __float_as_uint(m));
  }
}

// One thread per 1 x 16 group over the row-padded matrix; rows >= R only write a zero scale.
// amax_gs holds the tensor amax on entry; thread 0 of block 0 does not overwrite it (the
// per-tensor scale goes to gs_out).
template <typename T>
__global__ void nvfp4_quant_kernel(const T* __restrict__ x, int64_t R, int K, const float* __restrict__ amax,
                                   uint8_t* __restrict__ q, uint8_t* __restrict__ sf, float* __restrict__ gs_out) {
  const int groups = K / 16;
  const int64_t rows_pad = (R + 127) / 128 * 128;
  const int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (g >= rows_pad * groups) return;
  const int64_t r = g / groups;
  const int j = static_cast<int>(g % groups);
  const float gs = gscale_of(*amax);
  if (g == 0) *gs_out = gs;
  const int64_t so = sf_offset(r, j, K / 64);
  if (r >= R) {
    sf[so] = 0;
    return;
  }
  float v[16];
  load16(x + r * K + j * 16, v);
  float bmax = 0.f;
#pragma unroll
  for (int t = 0; t < 16; ++t) bmax = fmaxf(bmax, fabsf(v[t]));
  const uint8_t s8 = to_e4m3(fminf(bmax / 6.f / gs, 448.f));
  const float eff = from_e4m3(s8) * gs;
  const float inv = eff > 0.f ? 1.f / eff : 0.f;
  float lo[8], hi[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    lo[t] = v[t] * inv;
    hi[t] = v[8 + t] * inv;
  }
  uint2 packed;
  packed.x = pack_e2m1x8(lo);
  packed.y = pack_e2m1x8(hi);
  *reinterpret_cast<uint2*>(q + r * (K / 2) + j * 8) = packed;
  sf[so] = s8;
}

template <typename T>
__global__ void nvfp4_dequant_kernel(const uint8_t* __restrict__ q, const uint8_t* __restrict__ sf,
                                     const float* __restrict__ gs, int64_t R, int K, T* __restrict__ out) {
  const int groups = K / 16;
  const int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (g >= R * groups) return;
  const int64_t r = g / groups;
  const int j = static_cast<int>(g % groups);
  const float scale = from_e4m3(sf[sf_offset(r, j, K / 64)]) * (*gs);
  const uint2 packed = *reinterpret_cast<const uint2*>(q + r * (K / 2) + j * 8);
  const uint32_t w[2] = {packed.x, packed.y};
  T* o = out + r * K + j * 16;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float val = e2m1_value((w[h] >> (4 * t)) & 0xFu) * scale;
      if constexpr (std::is_same<T, float>::value)
        o[h * 8 + t] = val;
      else
        o[h * 8 + t] = __float2bfloat16(val);
    }
}

// ---------------------------------------------------------------- GEMM
struct Fp4GemmParams {
  int M, N, K;
  const uint8_t* sfa;  // blocked scales of A
  const uint8_t* sfb;  // blocked scales of B
  const float* gsa;
  const float* gsb;
  __nv_bfloat16* C;
  long ldc;
  const __nv_bfloat16* bias;
  int* status;
};

// Plain (non-tensor) bulk copy global -> shared, completing on an mbarrier. Both addresses
// 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory descriptor of one 512-byte scale block as the source of tcgen05.cp
// 32x128b: 32 rows of 16 bytes, no swizzle, 8-row core matrices 128 bytes apart (SBO).
__device__ __forceinline__ uint64_t make_sf_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(128u >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}

__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void umma_nvfp4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Instruction descriptor of a block-scaled MMA: A and B e2m1 (format 1 at bits 7-9 and
// 10-12), K-major, N >> 3 at bits 17-22, scale type ue4m3 (bit 23 = 0), M >> 4 at 24-28,
// scale-factor byte ids 0 (bits 4-5 and 29-30: four scales per 32-bit word), dense K = 64.
__host__ __device__ constexpr uint32_t make_idesc_nvfp4(int M, int N) {
  return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__global__ void __launch_bounds__(320, 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      Fp4GemmParams p) {
  using namespace fp4g;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accfull = empty + STAGES;
  uint64_t* accempty = accfull + 1;
  uint64_t* drain = accempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM, num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int nkt = p.K / BK;
  const int kblocks = p.K / 64;
  const int n_rowblocks = (p.N + 127) / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accfull, 1);
    mbar_init(accempty, 256);
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile % num_m, nb = tile / num_m;
        const bool second_half = 2 * nb + 1 < n_rowblocks;
        for (int kt = 0; kt < nkt; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + stage * STAGE_BYTES;
          uint8_t* sA = st;
          uint8_t* sB = sA + A_BYTES;
          uint8_t* sSFA = sB + B_BYTES;
          uint8_t* sSFB = sSFA + SFA_BYTES;
          mbar_expect_tx(&full[stage], A_BYTES + B_BYTES + SFA_BYTES + (second_half ? SFB_BYTES : SFB_BYTES / 2));
          tma_load_2d(sA, &tmA, &full[stage], kt * BKB, mb * BM);
          tma_load_2d(sB, &tmB, &full[stage], kt * BKB, nb * BN);
          tma_load_2d(sB + 128 * BKB, &tmB, &full[stage], kt * BKB, nb * BN + 128);
          bulk_load(sSFA, p.sfa + (static_cast<int64_t>(mb) * kblocks + kt * KK) * 512, SFA_BYTES, &full[stage]);
          bulk_load(sSFB, p.sfb + (static_cast<int64_t>(2 * nb) * kblocks + kt * KK) * 512, SFB_BYTES / 2,
                    &full[stage]);
          if (second_half)
            bulk_load(sSFB + SFB_BYTES / 2, p.sfb + (static_cast<int64_t>(2 * nb + 1) * kblocks + kt * KK) * 512,
                      SFB_BYTES / 2, &full[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = make_idesc_nvfp4(BM, BN);
      int stage = 0;
      uint32_t phase = 0, aphase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(accempty, aphase ^ 1, p.status, kStatusTimeoutMma)) break;
        aphase ^= 1;
        tc_fence_after();
        for (int kt = 0; kt < nkt; ++kt) {
          if (!mbar_wait(&full[stage], phase, p.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* st = smem + stage * STAGE_BYTES;
          const uint32_t a_base = smem_u32(st), b_base = smem_u32(st + A_BYTES);
          const uint32_t sfa_base = smem_u32(st + A_BYTES + B_BYTES);
          const uint32_t sfb_base = sfa_base + SFA_BYTES;
#pragma unroll
          for (int kk = 0; kk < KK; ++kk) {
            tmem_cp_sf(tmem_base + SFA_COL + 4 * kk, make_sf_desc(sfa_base + kk * 512));
            tmem_cp_sf(tmem_base + SFB_COL + 8 * kk, make_sf_desc(sfb_base + kk * 512));
            tmem_cp_sf(tmem_base + SFB_COL + 8 * kk + 4, make_sf_desc(sfb_base + SFB_BYTES / 2 + kk * 512));
          }
#pragma unroll
          for (int kk = 0; kk < KK; ++kk)
            umma_nvfp4(tmem_base, make_smem_desc_sw128(a_base + kk * 32, 16, 1024),
                       make_smem_desc_sw128(b_base + kk * 32, 16, 1024), IDESC, tmem_base + SFA_COL + 4 * kk,
                       tmem_base + SFB_COL + 8 * kk, (kt > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(accfull);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.status, kStatusTimeoutDrain);
    }
  } else {
    // Epilogue: lane quarter (warp % 4) -> rows; warps 2..5 columns 0..127, 6..9 columns 128..255.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const float alpha = __ldg(p.gsa) * __ldg(p.gsb);
    uint32_t aphase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int mb = tile % num_m, nb = tile / num_m;
      const bool got = mbar_wait(accfull, aphase, p.status, kStatusTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, got)) break;
      aphase ^= 1;
      tc_fence_after();
      float acc[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + lane_addr + half * 128 + c * 32, r);
#pragma unroll
        for (int t = 0; t < 32; ++t) acc[c * 32 + t] = __uint_as_float(r[t]);
      }
      tc_fence_before();
      mbar_arrive(accempty);
      const long m = static_cast<long>(mb) * BM + row;
      const int n0 = nb * BN + half * 128;
      if (m < p.M && n0 < p.N) {
        __nv_bfloat16* crow = p.C + m * p.ldc + n0;
#pragma unroll
        for (int c = 0; c < 128; c += 8) {
          if (n0 + c + 8 <= p.N) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              v[u] = acc[c + u] * alpha + (p.bias != nullptr ? __bfloat162float(p.bias[n0 + c + u]) : 0.f);
            uint4 o;
            o.x = pack_bf16x2(v[0], v[1]);
            o.y = pack_bf16x2(v[2], v[3]);
            o.z = pack_bf16x2(v[4], v[5]);
            o.w = pack_bf16x2(v[6], v[7]);
            *reinterpret_cast<uint4*>(crow + c) = o;
          } else {
            for (int u = 0; u < 8 && n0 + c + u < p.N; ++u)
              crow[c + u] = __float2bfloat16(acc[c + u] * alpha +
                                             (p.bias != nullptr ? __bfloat162float(p.bias[n0 + c + u]) : 0.f));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, fp4g::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host
int64_t nvfp4_sf_bytes(int64_t rows, int64_t cols) { return (rows + 127) / 128 * (cols / 64) * 512; }

// x [R, K] (bf16 or fp32, contiguous, K % 64 == 0) -> {q [R, K/2] uint8, sf (blocked) uint8, gs [1] fp32}.
std::vector<at::Tensor> nvfp4_quantize(const at::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "nvfp4_quantize: 2-D contiguous CUDA tensor");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat, "nvfp4_quantize: bf16 or fp32");
  const int64_t R = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 64 == 0 && K > 0, "nvfp4_quantize: K must be a positive multiple of 64");
  auto opts = x.options().dtype(at::kByte);
  at::Tensor q = at::empty({R, K / 2}, opts);
  at::Tensor sf = at::empty({nvfp4_sf_bytes(R, K)}, opts);
  at::Tensor amax = at::zeros({1}, x.options().dtype(at::kFloat));
  at::Tensor gs = at::empty({1}, x.options().dtype(at::kFloat));
  const int dev = x.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  const int64_t n16 = R * K / 16;
  const int64_t padded_groups = (R + 127) / 128 * 128 * (K / 16);
  if (n16 > 0) {
    const int blocks = static_cast<int>(std::min<int64_t>((n16 + 255) / 256, 4L * num_sms(dev)));
    if (x.scalar_type() == at::kBFloat16)
      nvfp4_amax_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), n16,
                                                    amax.data_ptr<float>());
    else
      nvfp4_amax_kernel<<<blocks, 256, 0, stream>>>(x.data_ptr<float>(), n16, amax.data_ptr<float>());
    NTB_LAUNCH_CHECK(1);
  }
  const int qblocks = static_cast<int>((padded_groups + 255) / 256);
  if (qblocks > 0) {
    if (x.scalar_type() == at::kBFloat16)
      nvfp4_quant_kernel<<<qblocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), R,
                                                      static_cast<int>(K), amax.data_ptr<float>(), q.data_ptr<uint8_t>(),
                                                      sf.data_ptr<uint8_t>(), gs.data_ptr<float>());
    else
      nvfp4_quant_kernel<<<qblocks, 256, 0, stream>>>(x.data_ptr<float>(), R, static_cast<int>(K),
                                                      amax.data_ptr<float>(), q.data_ptr<uint8_t>(),
                                                      sf.data_ptr<uint8_t>(), gs.data_ptr<float>());
    NTB_LAUNCH_CHECK(1);
  }
  return {q, sf, gs};
}

at::Tensor nvfp4_dequantize(const at::Tensor& q, const at::Tensor& sf, const at::Tensor& gs, at::ScalarType dtype) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 2 && q.is_contiguous() && q.scalar_type() == at::kByte,
              "nvfp4_dequantize: packed uint8 [R, K/2]");
  const int64_t R = q.size(0), K = q.size(1) * 2;
  TORCH_CHECK(K % 64 == 0, "nvfp4_dequantize: K must be a multiple of 64");
  TORCH_CHECK(sf.scalar_type() == at::kByte && sf.numel() == nvfp4_sf_bytes(R, K), "nvfp4_dequantize: scale blocks");
  TORCH_CHECK(gs.scalar_type() == at::kFloat && gs.numel() == 1, "nvfp4_dequantize: fp32 tensor scale");
  TORCH_CHECK(dtype == at::kBFloat16 || dtype == at::kFloat, "nvfp4_dequantize: bf16 or fp32 output");
  at::Tensor out = at::empty({R, K}, q.options().dtype(dtype));
  const int64_t n = R * (K / 16);
  if (n == 0) return out;
  const int dev = q.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  const int blocks = static_cast<int>((n + 255) / 256);
  if (dtype == at::kBFloat16)
    nvfp4_dequant_kernel<<<blocks, 256, 0, stream>>>(q.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>(),
                                                     gs.data_ptr<float>(), R, static_cast<int>(K),
                                                     reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  else
    nvfp4_dequant_kernel<<<blocks, 256, 0, stream>>>(q.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>(),
                                                     gs.data_ptr<float>(), R, static_cast<int>(K), out.data_ptr<float>());
  NTB_LAUNCH_CHECK(1);
  return out;
}

// out[M, N] (bf16) = dequant(a) . dequant(b)^T (+ bias) on the e2m1 tensor cores.
void gemm_nvfp4(const at::Tensor& a_q, const at::Tensor& sfa, const at::Tensor& gsa, const at::Tensor& b_q,
                const at::Tensor& sfb, const at::Tensor& gsb, at::Tensor& out, const c10::optional<at::Tensor>& bias) {
  using namespace fp4g;
  TORCH_CHECK(a_q.is_cuda() && b_q.is_cuda() && a_q.scalar_type() == at::kByte && b_q.scalar_type() == at::kByte,
              "gemm_nvfp4: packed e2m1 operands as uint8 CUDA tensors");
  TORCH_CHECK(a_q.dim() == 2 && b_q.dim() == 2 && a_q.is_contiguous() && b_q.is_contiguous(),
              "gemm_nvfp4: 2-D contiguous operands");
  const int64_t M = a_q.size(0), K = a_q.size(1) * 2, N = b_q.size(0);
  TORCH_CHECK(b_q.size(1) * 2 == K && K % BK == 0 && K > 0, "gemm_nvfp4: K must match and be a multiple of 256");
  TORCH_CHECK(sfa.scalar_type() == at::kByte && sfa.numel() == nvfp4_sf_bytes(M, K), "gemm_nvfp4: A scale blocks");
  TORCH_CHECK(sfb.scalar_type() == at::kByte && sfb.numel() == nvfp4_sf_bytes(N, K), "gemm_nvfp4: B scale blocks");
  TORCH_CHECK(gsa.scalar_type() == at::kFloat && gsa.numel() == 1 && gsb.scalar_type() == at::kFloat &&
                  gsb.numel() == 1,
              "gemm_nvfp4: fp32 tensor scales");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(sfa.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(sfb.data_ptr()) & 15) == 0,
              "gemm_nvfp4: scale blocks must be 16-byte aligned");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1 &&
                  out.stride(0) % 8 == 0,
              "gemm_nvfp4: bf16 out [M, N] with 16-byte aligned rows");
  TORCH_CHECK(N % 8 == 0, "gemm_nvfp4: N multiple of 8");
  if (bias.has_value())
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N, "gemm_nvfp4: bias bf16 [N]");
  if (M == 0 || N == 0) return;
  Fp4GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.sfa = sfa.data_ptr<uint8_t>();
  p.sfb = sfb.data_ptr<uint8_t>();
  p.gsa = gsa.data_ptr<float>();
  p.gsb = gsb.data_ptr<float>();
  p.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldc = out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  const int dev = a_q.get_device();
  p.status = device_status(dev);
  TmaSlots& ts = tls_tma_slots();
  make_tma_2d(&ts.m[0], a_q.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, M, K / 2, BKB, 128,
              CU_TENSOR_MAP_SWIZZLE_128B);
  make_tma_2d(&ts.m[1], b_q.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, K / 2, BKB, 128,
              CU_TENSOR_MAP_SWIZZLE_128B);
  static bool attr_done[64] = {};
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    NTB_CUDA_CHECK(cudaFuncSetAttribute(gemm_nvfp4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr_done[dev] = true;
  }
  const int tiles = static_cast<int>(((M + BM - 1) / BM) * ((N + BN - 1) / BN));
  const int grid = std::min(tiles, num_sms(dev));
  void* args[3] = {&ts.m[0], &ts.m[1], &p};
  NTB_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(gemm_nvfp4_kernel), dim3(grid), dim3(THREADS), args,
                                  static_cast<size_t>(SMEM_BYTES), at::cuda::getCurrentCUDAStream(dev)));
  NTB_LAUNCH_CHECK(1);
}

}  // namespace ntb
