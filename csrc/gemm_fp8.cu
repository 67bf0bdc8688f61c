// Block-scaled fp8 (e4m3) GEMM on the 5th-generation tensor cores (sm_100a), the
// DeepSeek-V3 recipe:
//
//   C[M, N] = sum_kb ( A_q[:, kb] . B_q[:, kb]^T ) * sa[m, kb] * sb[n / 128, kb]   (+ bias)
//
// A_q: e4m3 [M, K] (activations, one fp32 scale per row and 128-column tile, sa [M, K/128]),
// B_q: e4m3 [N, K] (weights, one fp32 scale per 128 x 128 block, sb [ceil(N/128), K/128]),
// both K-major, K a multiple of 128; C bf16. The scales are exactly what the e4m3
// quantizer in quant.cu produces (tile_1x128 / block_128x128).
//
// Persistent CTAs, 320 threads, 128 x 256 output tiles (a 256-wide B tile halves the shared-
// memory operand traffic per FLOP relative to 128, which the doubled fp8 rate needs):
//   warp 0      TMA producer: per K block one [128 x 128 B] box of A and two of B (128-byte
//               swizzle: one swizzle row = one 128-wide K block of 8-bit elements)
//   warp 1      MMA issuer: 4 x tcgen05.mma kind::f8f6f4 (128 x 256 x 32) per K block into
//               one of two TMEM partial buffers (fresh accumulation per K block)
//   warps 2..9  promotion: two warps per TMEM lane quarter (32 rows), each owning one
//               128-column half = one weight-scale block; per K block they read the partial
//               product, scale it by sa[row, kb] * sb[block, kb] and add it to fp32
//               registers, then release the buffer, so the tensor core computes K block k+1
//               while block k is promoted; after the last K block they add the bias and
//               store bf16.
// Every wait is bounded (common.cuh).
//
// Reference parity: src/runtime/te_backend.py:229-260 (emulated fp8 linear: fake-quantised
// operands, fp32 GEMM) with the recipe of src/runtime/mixed_precision.py:222-291.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace ntb {

namespace fp8g {
constexpr int BM = 128, BN = 256, BK = 128;  // BK in elements = bytes; BN = two weight-scale blocks
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK;
constexpr int SMEM_BYTES = 1024 + STAGES * (A_BYTES + B_BYTES) + 512;
constexpr int THREADS = 320;
constexpr int NBUF = 2;              // TMEM partial buffers of BN columns (the tensor core runs a K block ahead)
constexpr uint32_t TMEM_COLS = NBUF * BN;
}  // namespace fp8g

struct Fp8GemmParams {
  int M, N, K;
  const float* sa;  // [M, K/128]
  const float* sb;  // [ceil(N/128), K/128], or for grouped B [groups * N / 128, K/128]
  __nv_bfloat16* C;
  long ldc;
  const __nv_bfloat16* bias;
  int* status;
  // M-grouped mode (offsets != nullptr): the rows of A and C are expert segments, each padded to a
  // multiple of 128 rows ([offsets[g], offsets[g+1])); B is a stack of per-expert [N, K] matrices.
  const int* offsets;
  int groups;
};

// Expert of the 128-row tile starting at `row`, or -1 beyond the last segment (tile skipped).
__device__ __forceinline__ int fp8_group_of_tile(const Fp8GemmParams& p, int row) {
  if (p.offsets == nullptr) return 0;
  if (row >= __ldg(p.offsets + p.groups)) return -1;
  int lo = 0, hi = p.groups - 1;  // last g with offsets[g] <= row
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(p.offsets + mid) <= row) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void umma_f8f6f4_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::f8f6f4: f32 accumulator (bits 4-5 = 1), A and B e4m3
// (format code 0 at bits 7-9 and 10-12), both K-major, N >> 3 at 17, M >> 4 at 24.
__host__ __device__ constexpr uint32_t make_idesc_e4m3(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__global__ void __launch_bounds__(320, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    Fp8GemmParams p) {
  using namespace fp8g;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* pfull = empty + STAGES;  // [NBUF]
  uint64_t* pempty = pfull + NBUF;   // [NBUF]
  uint64_t* drain = pempty + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM, num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int nkb = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 256);
    }
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
        const int g = fp8_group_of_tile(p, mb * BM);
        if (g < 0) continue;
        const int b0 = g * p.N + nb * BN;  // first B row of this tile (this expert's slice)
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, mb * BM);
          tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * BK, b0);
          tma_load_2d(sB + stage * B_BYTES + 128 * BK, &tmB, &full[stage], kb * BK, b0 + 128);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = make_idesc_e4m3(BM, BN);
      int stage = 0, buf = 0;
      uint32_t phase = 0, bphase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (fp8_group_of_tile(p, (tile % num_m) * BM) < 0) continue;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&pempty[buf], bphase ^ 1, p.status, kStatusTimeoutMma) ||
              !mbar_wait(&full[stage], phase, p.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_BYTES), b_base = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            umma_f8f6f4_ss(tmem_base + buf * BN, make_smem_desc_sw128(a_base + k * 32, 16, 1024),
                           make_smem_desc_sw128(b_base + k * 32, 16, 1024), IDESC, k > 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          umma_commit(&pfull[buf]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if (++buf == NBUF) {
            buf = 0;
            bphase ^= 1;
          }
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // Promotion warps: lane quarter (warp % 4) -> rows; warps 2..5 columns 0..127, 6..9 columns 128..255.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const int nk = p.K / BK;
    int buf = 0;
    uint32_t bphase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int mb = tile % num_m, nb = tile / num_m;
      const int g = fp8_group_of_tile(p, mb * BM);
      if (g < 0) continue;
      const long m = static_cast<long>(mb) * BM + row;
      const float* sa_row = p.sa + (m < p.M ? m : 0) * nk;
      // this half's weight block (for a stacked B, inside expert g's slice of N / 128 blocks)
      const float* sb_row = p.sb + (static_cast<long>(g) * (p.N / 128) + nb * 2 + half) * nk;
      const bool half_live = nb * BN + half * 128 < p.N;
      float acc[128];
#pragma unroll
      for (int c = 0; c < 128; ++c) acc[c] = 0.f;
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        const float sc = half_live ? __ldg(sa_row + kb) * __ldg(sb_row + kb) : 0.f;
        const bool got = mbar_wait(&pfull[buf], bphase, p.status, kStatusTimeoutEpilogue);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem_base + lane_addr + buf * BN + half * 128 + c * 32, r);
#pragma unroll
          for (int t = 0; t < 32; ++t) acc[c * 32 + t] = fmaf(__uint_as_float(r[t]), sc, acc[c * 32 + t]);
        }
        tc_fence_before();
        mbar_arrive(&pempty[buf]);
        if (++buf == NBUF) {
          buf = 0;
          bphase ^= 1;
        }
      }
      if (!ok) break;
      const int n0 = nb * BN + half * 128;
      if (m < p.M && half_live) {
        __nv_bfloat16* crow = p.C + m * p.ldc + n0;
#pragma unroll
        for (int c = 0; c < 128; c += 8) {
          if (n0 + c + 8 <= p.N) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              v[u] = acc[c + u] + (p.bias != nullptr ? __bfloat162float(p.bias[n0 + c + u]) : 0.f);
            uint4 o;
            o.x = pack_bf16x2(v[0], v[1]);
            o.y = pack_bf16x2(v[2], v[3]);
            o.z = pack_bf16x2(v[4], v[5]);
            o.w = pack_bf16x2(v[6], v[7]);
            *reinterpret_cast<uint4*>(crow + c) = o;
          } else {
            for (int u = 0; u < 8 && n0 + c + u < p.N; ++u)
              crow[c + u] = __float2bfloat16(acc[c + u] + (p.bias != nullptr ? __bfloat162float(p.bias[n0 + c + u]) : 0.f));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, fp8g::TMEM_COLS);
  }
}

static void launch_fp8(const at::Tensor& a_q, const at::Tensor& b_q, Fp8GemmParams& p, int64_t b_rows) {
  using namespace fp8g;
  const int dev = a_q.get_device();
  p.status = device_status(dev);
  TmaSlots& ts = tls_tma_slots();
  make_tma_2d(&ts.m[0], a_q.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.K, p.M, p.K, 128, 128,
              CU_TENSOR_MAP_SWIZZLE_128B);
  make_tma_2d(&ts.m[1], b_q.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.K, b_rows, p.K, 128, 128,
              CU_TENSOR_MAP_SWIZZLE_128B);
  static bool attr_done[64] = {};
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    NTB_CUDA_CHECK(cudaFuncSetAttribute(gemm_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr_done[dev] = true;
  }
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  const int grid = std::min(tiles, num_sms(dev));
  void* args[3] = {&ts.m[0], &ts.m[1], &p};
  NTB_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(gemm_fp8_kernel), dim3(grid), dim3(THREADS), args,
                                  static_cast<size_t>(SMEM_BYTES), at::cuda::getCurrentCUDAStream(dev)));
  NTB_LAUNCH_CHECK(1);
}

// Grouped (mixture-of-experts) form: out[rows of g] = a_q[rows of g] . b_q[g]^T with per-row 1x128
// activation scales and 128x128 block scales of the stacked weights. a_q: e4m3 [R, K] whose rows are
// expert segments padded to multiples of 128 (offsets int32 [G + 1], device, as the bf16 grouped
// GEMM takes them); b_q: e4m3 [G * N, K]; sb: [G * N / 128, K / 128]; out bf16 [R, N]. Rows of out
// beyond offsets[G] are not written.
void gemm_fp8_grouped(const at::Tensor& a_q, const at::Tensor& sa, const at::Tensor& b_q, const at::Tensor& sb,
                      at::Tensor& out, const at::Tensor& offsets) {
  TORCH_CHECK(a_q.is_cuda() && b_q.is_cuda() && a_q.scalar_type() == at::kByte && b_q.scalar_type() == at::kByte &&
                  a_q.is_contiguous() && b_q.is_contiguous() && a_q.dim() == 2 && b_q.dim() == 2,
              "gemm_fp8_grouped: contiguous 2-D e4m3 operands (uint8)");
  TORCH_CHECK(offsets.is_cuda() && offsets.scalar_type() == at::kInt && offsets.is_contiguous() && offsets.numel() >= 2,
              "gemm_fp8_grouped: int32 offsets [G + 1]");
  const int64_t R = a_q.size(0), K = a_q.size(1), G = offsets.numel() - 1;
  TORCH_CHECK(b_q.size(1) == K && K % 128 == 0 && R % 128 == 0 && b_q.size(0) % G == 0,
              "gemm_fp8_grouped: K multiple of 128, rows padded to 128, stacked B rows divisible by G");
  const int64_t N = b_q.size(0) / G;
  TORCH_CHECK(N % 128 == 0, "gemm_fp8_grouped: per-expert N must be a multiple of 128");
  TORCH_CHECK(sa.scalar_type() == at::kFloat && sa.is_contiguous() && sa.size(0) == R && sa.size(1) == K / 128,
              "gemm_fp8_grouped: activation scales [R, K/128]");
  TORCH_CHECK(sb.scalar_type() == at::kFloat && sb.is_contiguous() && sb.size(0) == G * N / 128 && sb.size(1) == K / 128,
              "gemm_fp8_grouped: weight scales [G * N / 128, K/128]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(0) == R && out.size(1) == N && out.stride(1) == 1,
              "gemm_fp8_grouped: bf16 out [R, N]");
  if (R == 0) return;
  Fp8GemmParams p{};
  p.M = static_cast<int>(R);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.sa = sa.data_ptr<float>();
  p.sb = sb.data_ptr<float>();
  p.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldc = out.stride(0);
  p.offsets = offsets.data_ptr<int>();
  p.groups = static_cast<int>(G);
  launch_fp8(a_q, b_q, p, G * N);
}

// out[M, N] (bf16) = dequant(a_q, sa) . dequant(b_q, sb)^T (+ bias), computed on the e4m3 operands.
void gemm_fp8_blockscaled(const at::Tensor& a_q, const at::Tensor& sa, const at::Tensor& b_q, const at::Tensor& sb,
                          at::Tensor& out, const c10::optional<at::Tensor>& bias) {
  using namespace fp8g;
  TORCH_CHECK(a_q.is_cuda() && b_q.is_cuda() && a_q.scalar_type() == at::kByte && b_q.scalar_type() == at::kByte,
              "gemm_fp8: e4m3 operands as uint8 CUDA tensors");
  TORCH_CHECK(a_q.dim() == 2 && b_q.dim() == 2 && a_q.is_contiguous() && b_q.is_contiguous(), "gemm_fp8: 2-D contiguous");
  const int64_t M = a_q.size(0), K = a_q.size(1), N = b_q.size(0);
  TORCH_CHECK(b_q.size(1) == K && K % 128 == 0, "gemm_fp8: K must match and be a multiple of 128");
  TORCH_CHECK(sa.scalar_type() == at::kFloat && sa.is_contiguous() && sa.size(0) == M && sa.size(1) == K / 128,
              "gemm_fp8: activation scales [M, K/128]");
  TORCH_CHECK(sb.scalar_type() == at::kFloat && sb.is_contiguous() && sb.size(0) == (N + 127) / 128 &&
                  sb.size(1) == K / 128,
              "gemm_fp8: weight scales [ceil(N/128), K/128]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1,
              "gemm_fp8: bf16 out [M, N]");
  TORCH_CHECK(N % 8 == 0, "gemm_fp8: N multiple of 8");
  if (bias.has_value())
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N, "gemm_fp8: bias bf16 [N]");
  if (M == 0 || N == 0) return;
  Fp8GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.sa = sa.data_ptr<float>();
  p.sb = sb.data_ptr<float>();
  p.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldc = out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  launch_fp8(a_q, b_q, p, N);
}

}  // namespace ntb
