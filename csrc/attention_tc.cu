// Causal / full flash attention forward on the 5th-generation tensor cores (sm_100a).
//
// Head dim 128 for Q, K and V; GQA by head-index mapping; q/k/v are [B, S, H, 128]
// views with arbitrary 16-byte-aligned strides (e.g. slices of a fused QKV
// projection), addressed through 4-D TMA tensor maps (d, s, h, b). Outputs match
// flash_attn_fwd in attention.cu: o [B, S, Hq, 128] bf16 and lse [B, Hq, S] fp32
// in the log2 domain (m + log2(l) of the scores scaled by softmax_scale * log2 e),
// so the existing backward consumes them unchanged.
//
// One CTA per (128-query tile, head, batch), 192 threads:
//   warp 0      TMA producer: Q once, then K_j / V_j blocks of 128 keys through
//               two 2-stage rings (each tile = two 16 KB boxes of [128 rows x 64]
//               elements, 128-byte swizzle)
//   warp 1      MMA issuer (one thread) and TMEM owner (512 columns):
//               S_j = Q K_j^T into TMEM buffer j % 2 (columns 0 / 128), and
//               O += P_j V_j into TMEM columns 256..383; issue order
//               S_0, S_1, PV_0, S_2, PV_1, ... so S_{j+1} runs on the tensor
//               core while the softmax works on S_j
//   warps 2..5  softmax, one thread per query row (TMEM lane): tcgen05.ld of the
//               row of S_j, scale/mask, row max, exp2, row sum; P_j written as bf16
//               into shared memory in the 128-byte-swizzled K-major layout the MMA
//               descriptor expects; online-softmax correction of O in TMEM only
//               when the running max grows by more than 2^8 (otherwise the stale
//               max is kept: P <= 256, exact after the final division); epilogue
//               O / l and lse.
// Every wait is bounded (common.cuh) and reports through the status word.
//
// Reference parity: src/models/attention.py:134-220 and src/models/deepseek.py:681-738
// compute softmax(QK^T * scale + causal mask) V with materialised fp32 scores.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace ntb {

namespace attn_tc {

constexpr int BM = 128, BN = 128, D = 128;
constexpr int TILE_BYTES = BM * D * 2;          // 32 KB: two [128 x 64] swizzled boxes
constexpr int BOX_BYTES = TILE_BYTES / 2;       // 16 KB
constexpr int SMEM_Q = 0;
constexpr int SMEM_K = SMEM_Q + TILE_BYTES;     // 2 stages
constexpr int SMEM_V = SMEM_K + 2 * TILE_BYTES; // 2 stages
constexpr int SMEM_P = SMEM_V + 2 * TILE_BYTES;
constexpr int SMEM_BAR = SMEM_P + TILE_BYTES;
constexpr int SMEM_BYTES = 1024 + SMEM_BAR + 256;
constexpr uint32_t TMEM_COLS = 512, TMEM_S0 = 0, TMEM_O = 256;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

// 2^x on the special-function unit (PTX ex2.approx, flushes subnormal results to 0;
// relative error far below bf16 resolution, which is what P is stored in).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Every lane waits (bounded); the outcome is made warp-uniform so that the
// .sync.aligned tcgen05 loads/stores that follow are never executed by part of a warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  const bool ok = mbar_wait(bar, parity, status, code);
  return __all_sync(0xffffffffu, ok);
}

}  // namespace attn_tc

struct AttnTcParams {
  __nv_bfloat16* o;
  float* lse;
  int B, S, Hq, Hkv;
  float scale_log2;
  int causal;
  int* status;
};

__global__ void __launch_bounds__(192, 1)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, AttnTcParams p) {
  using namespace attn_tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_free = bars + 11;  // [2]
  uint64_t* p_full = bars + 13;
  uint64_t* o_done = bars + 14;
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int q0 = qb * BM;
  const int nkb_all = (p.S + BN - 1) / BN;
  const int nkb = p.causal ? min(nkb_all, qb + 1) : nkb_all;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
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
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_expect_tx(q_full, TILE_BYTES);
      for (int c = 0; c < 2; ++c) tma_load_4d(smem + SMEM_Q + c * BOX_BYTES, &tmQ, q_full, c * 64, q0, h, b);
      for (int j = 0; j < nkb; ++j) {
        const int st = j & 1;
        const uint32_t ph = static_cast<uint32_t>((j >> 1) & 1);
        if (!mbar_wait(&k_empty[st], ph ^ 1, p.status, kStatusTimeoutProducer)) break;
        mbar_expect_tx(&k_full[st], TILE_BYTES);
        for (int c = 0; c < 2; ++c)
          tma_load_4d(smem + SMEM_K + st * TILE_BYTES + c * BOX_BYTES, &tmK, &k_full[st], c * 64, j * BN, hk, b);
        if (!mbar_wait(&v_empty[st], ph ^ 1, p.status, kStatusTimeoutProducer)) break;
        mbar_expect_tx(&v_full[st], TILE_BYTES);
        for (int c = 0; c < 2; ++c)
          tma_load_4d(smem + SMEM_V + st * TILE_BYTES + c * BOX_BYTES, &tmV, &v_full[st], c * 64, j * BN, hk, b);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = make_idesc_f16(BM, BN, false, false);  // Q K-major, K K-major
      constexpr uint32_t IDESC_O = make_idesc_f16(BM, D, false, true);    // P K-major, V N-major
      const uint32_t sQ = smem_u32(smem + SMEM_Q), sP = smem_u32(smem + SMEM_P);
      bool ok = mbar_wait(q_full, 0, p.status, kStatusTimeoutMma);
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait(p_full, static_cast<uint32_t>(i & 1), p.status, kStatusTimeoutMma)) return false;
        const int st = i & 1;
        if (!mbar_wait(&v_full[st], static_cast<uint32_t>((i >> 1) & 1), p.status, kStatusTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t sV = smem_u32(smem + SMEM_V + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // A = P [128 q x 128 keys] K-major: 64-key chunks 16 KB apart, 32 B per k16 step inside.
          const uint64_t adesc = make_smem_desc_sw128(sP + (kk >> 2) * BOX_BYTES + (kk & 3) * 32, 16, 1024);
          // B = V as [keys][dv] (N-major): 64-dv chunks 16 KB apart (LBO), k16 step = 16 key rows.
          const uint64_t bdesc = make_smem_desc_sw128(sV + kk * 2048, BOX_BYTES, 1024);
          umma_f16_ss(tmem_base + TMEM_O, adesc, bdesc, IDESC_O, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(o_done);
        umma_commit(&v_empty[st]);
        return true;
      };
      for (int j = 0; ok && j < nkb; ++j) {
        const int st = j & 1;
        const uint32_t ph = static_cast<uint32_t>((j >> 1) & 1);
        if (!mbar_wait(&k_full[st], ph, p.status, kStatusTimeoutMma)) break;
        if (!mbar_wait(&s_free[st], ph ^ 1, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        const uint32_t sK = smem_u32(smem + SMEM_K + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * BOX_BYTES + (kk & 3) * 32;
          umma_f16_ss(tmem_base + TMEM_S0 + st * BN, make_smem_desc_sw128(sQ + off, 16, 1024),
                      make_smem_desc_sw128(sK + off, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && nkb > 0) issue_pv(nkb - 1);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;
    const int row = q0 + r_local;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* sP = smem + SMEM_P;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int st = j & 1;
      if (!warp_wait(&s_full[st], static_cast<uint32_t>((j >> 1) & 1), p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = tmem_base + lane_addr + TMEM_S0 + st * BN;
      const int key0 = j * BN;
      const bool need_mask = (key0 + BN > p.S) || (p.causal && key0 + BN - 1 > q0);
      // Columns t <= lim of this row are valid (causal: key <= row; tail: key < S).
      int lim = BN - 1;
      if (need_mask) {
        lim = min(lim, p.S - 1 - key0);
        if (p.causal) lim = min(lim, row - key0);
      }
      // Pass 1: row max of the raw scores (scale > 0 keeps the order), four independent chains.
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(s_addr + c * 32, r);
        if (need_mask) {
#pragma unroll
          for (int t = 0; t < 32; ++t)
            if (c * 32 + t <= lim) mx4[t & 3] = fmaxf(mx4[t & 3], __uint_as_float(r[t]));
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) mx4[t & 3] = fmaxf(mx4[t & 3], __uint_as_float(r[t]));
        }
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
      const float m_new = fmaxf(m, mx);
      // Lazy rescale: move this row's base only when its max grew by more than the threshold
      // (alpha is then < 2^-8); rows that keep their base get alpha = 1.
      const bool first = (m == -INFINITY);
      const bool rescale = first || (m_new > m + RESCALE_THRESHOLD);
      const float m_use = rescale ? (m_new == -INFINITY ? 0.f : m_new) : m;
      const float alpha = first ? 0.f : ex2_approx(m - m_use);
      if (j > 0 && !warp_wait(o_done, static_cast<uint32_t>((j - 1) & 1), p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      // Pass 2: p = 2^(s * scale_log2 - m), row sum, bf16 P into shared memory (swizzled K-major).
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
      const float neg_m = -m_use;
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(s_addr + c * 32, r);
        float pv[32];
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          float e = ex2_approx(fmaf(__uint_as_float(r[t]), p.scale_log2, neg_m));
          if (need_mask && c * 32 + t > lim) e = 0.f;
          pv[t] = e;
          sum4[t & 3] += e;
        }
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          uint4 v;
          v.x = pack_bf16x2(pv[q8 * 8 + 0], pv[q8 * 8 + 1]);
          v.y = pack_bf16x2(pv[q8 * 8 + 2], pv[q8 * 8 + 3]);
          v.z = pack_bf16x2(pv[q8 * 8 + 4], pv[q8 * 8 + 5]);
          v.w = pack_bf16x2(pv[q8 * 8 + 6], pv[q8 * 8 + 7]);
          const int chunk16 = c * 4 + q8;  // 16-byte chunk index along the 128 keys
          const int kc = chunk16 >> 3, j16 = chunk16 & 7;
          *reinterpret_cast<uint4*>(sP + kc * BOX_BYTES + r_local * 128 + ((j16 ^ (r_local & 7)) << 4)) = v;
        }
      }
      tc_fence_before();
      mbar_arrive(&s_free[st]);  // S buffer consumed (both passes done)
      const float rowsum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
      // O correction (warp-uniform: any lane of the warp that moved its base).
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          const uint32_t ta = tmem_base + lane_addr + TMEM_O + c * 32;
          tmem_ld32(ta, r);
#pragma unroll
          for (int t = 0; t < 32; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
          tmem_st32(ta, r);
        }
        tmem_wait_st();
      }
      l = first ? rowsum : l * alpha + rowsum;
      m = m_use;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P (generic writes) -> tensor core reads
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && nkb > 0 && warp_wait(o_done, static_cast<uint32_t>((nkb - 1) & 1), p.status, kStatusTimeoutEpilogue)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool valid = row < p.S;
      __nv_bfloat16* og = p.o + ((static_cast<int64_t>(b) * p.S + (valid ? row : 0)) * p.Hq + h) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + lane_addr + TMEM_O + c * 32, r);  // whole warp; stores below are per row
        if (valid) {
#pragma unroll
          for (int t = 0; t < 32; t += 8) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(r[t + 0]) * inv, __uint_as_float(r[t + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(r[t + 2]) * inv, __uint_as_float(r[t + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(r[t + 4]) * inv, __uint_as_float(r[t + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(r[t + 6]) * inv, __uint_as_float(r[t + 7]) * inv);
            *reinterpret_cast<uint4*>(og + c * 32 + t) = v;
          }
        }
      }
      if (valid) p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.S + row] = m + log2f(l);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// q, k, v: [B, S, H, 128] bf16 views (head dim contiguous, 16-byte aligned strides).
std::vector<at::Tensor> flash_attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                                          bool causal) {
  using namespace attn_tc;
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "flash_attn_fwd_tc: [B, S, H, D] tensors");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "flash_attn_fwd_tc: bf16");
  TORCH_CHECK(q.size(3) == D && k.size(3) == D && v.size(3) == D, "flash_attn_fwd_tc: head dim 128");
  TORCH_CHECK(q.stride(3) == 1 && k.stride(3) == 1 && v.stride(3) == 1, "flash_attn_fwd_tc: head dim contiguous");
  TORCH_CHECK(k.size(1) == q.size(1) && v.size(1) == q.size(1) && k.size(0) == q.size(0) && v.size(0) == q.size(0),
              "flash_attn_fwd_tc: self-attention shapes");
  TORCH_CHECK(q.size(2) % k.size(2) == 0 && k.size(2) == v.size(2), "flash_attn_fwd_tc: GQA head ratio");
  const int64_t B = q.size(0), S = q.size(1), Hq = q.size(2), Hkv = k.size(2);
  auto o = at::empty({B, S, Hq, D}, q.options());
  auto lse = at::empty({B, Hq, S}, q.options().dtype(at::kFloat));
  if (S == 0 || B == 0) return {o, lse};
  AttnTcParams p{};
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.Hq = static_cast<int>(Hq);
  p.Hkv = static_cast<int>(Hkv);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  const int dev = q.get_device();
  p.status = device_status(dev);
  TmaSlots& ts = tls_tma_slots();
  const int box[4] = {64, BM, 1, 1};
  {
    const int64_t dims[4] = {D, S, Hq, B};
    const int64_t str[3] = {q.stride(1), q.stride(2), q.stride(0)};
    make_tma_4d_bf16(&ts.m[0], q.data_ptr(), dims, str, box);
  }
  {
    const int64_t dims[4] = {D, S, Hkv, B};
    const int64_t str[3] = {k.stride(1), k.stride(2), k.stride(0)};
    make_tma_4d_bf16(&ts.m[1], k.data_ptr(), dims, str, box);
  }
  {
    const int64_t dims[4] = {D, S, Hkv, B};
    const int64_t str[3] = {v.stride(1), v.stride(2), v.stride(0)};
    make_tma_4d_bf16(&ts.m[2], v.data_ptr(), dims, str, box);
  }
  static bool attr_done[64] = {};
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    NTB_CUDA_CHECK(cudaFuncSetAttribute(flash_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr_done[dev] = true;
  }
  dim3 grid(static_cast<unsigned>((S + BM - 1) / BM), static_cast<unsigned>(Hq), static_cast<unsigned>(B));
  void* args[4] = {&ts.m[0], &ts.m[1], &ts.m[2], &p};
  NTB_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(flash_fwd_tc_kernel), grid, dim3(192), args,
                                  static_cast<size_t>(SMEM_BYTES), at::cuda::getCurrentCUDAStream(dev)));
  NTB_LAUNCH_CHECK(1);
  return {o, lse};
}

}  // namespace ntb
