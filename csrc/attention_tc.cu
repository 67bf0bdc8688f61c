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

constexpr int BM = 128, BN = 128;
constexpr int BOX_BYTES = BM * 64 * 2;          // 16 KB: one [128 rows x 64] swizzled box
constexpr uint32_t TMEM_COLS = 512, TMEM_S0 = 0, TMEM_O = 256;

// Shared-memory plan of the forward for head dims DQK (q, k) and DV (v, o), with KS K stages and VS V
// stages: Q (DQK/64 boxes), K ring, V ring, P (two boxes: 128 keys), barriers.
template <int DQK, int DV, int KS, int VS>
struct FwdCfg {
  static_assert(DQK % 64 == 0 && DV % 64 == 0 && DQK <= 192 && DV <= 128, "head dims");
  static constexpr int QB = DQK / 64, VB = DV / 64;
  static constexpr int Q_BYTES = QB * BOX_BYTES, V_BYTES = VB * BOX_BYTES;
  static constexpr int SMEM_Q = 0;
  static constexpr int SMEM_K = SMEM_Q + Q_BYTES;
  static constexpr int SMEM_V = SMEM_K + KS * Q_BYTES;
  static constexpr int SMEM_P = SMEM_V + VS * V_BYTES;
  static constexpr int SMEM_BAR = SMEM_P + 2 * BOX_BYTES;
  static constexpr int SMEM_BYTES = 1024 + SMEM_BAR + 256;
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};
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

template <int DQK, int DV, int KS, int VS>
__global__ void __launch_bounds__(192, 1)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, AttnTcParams p) {
  using namespace attn_tc;
  using Cfg = FwdCfg<DQK, DV, KS, VS>;
  constexpr int SMEM_Q = Cfg::SMEM_Q, SMEM_K = Cfg::SMEM_K, SMEM_V = Cfg::SMEM_V, SMEM_P = Cfg::SMEM_P,
                SMEM_BAR = Cfg::SMEM_BAR;
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
    }  // rings with one stage use entry 0 only
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
      mbar_expect_tx(q_full, Cfg::Q_BYTES);
      for (int c = 0; c < Cfg::QB; ++c) tma_load_4d(smem + SMEM_Q + c * BOX_BYTES, &tmQ, q_full, c * 64, q0, h, b);
      for (int j = 0; j < nkb; ++j) {
        const int st = j % KS, sv = j % VS;
        const uint32_t ph = static_cast<uint32_t>((j / KS) & 1), phv = static_cast<uint32_t>((j / VS) & 1);
        if (!mbar_wait(&k_empty[st], ph ^ 1, p.status, kStatusTimeoutProducer)) break;
        mbar_expect_tx(&k_full[st], Cfg::Q_BYTES);
        for (int c = 0; c < Cfg::QB; ++c)
          tma_load_4d(smem + SMEM_K + st * Cfg::Q_BYTES + c * BOX_BYTES, &tmK, &k_full[st], c * 64, j * BN, hk, b);
        if (!mbar_wait(&v_empty[sv], phv ^ 1, p.status, kStatusTimeoutProducer)) break;
        mbar_expect_tx(&v_full[sv], Cfg::V_BYTES);
        for (int c = 0; c < Cfg::VB; ++c)
          tma_load_4d(smem + SMEM_V + sv * Cfg::V_BYTES + c * BOX_BYTES, &tmV, &v_full[sv], c * 64, j * BN, hk, b);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_S = make_idesc_f16(BM, BN, false, false);  // Q K-major, K K-major
      constexpr uint32_t IDESC_O = make_idesc_f16(BM, DV, false, true);   // P K-major, V N-major
      const uint32_t sQ = smem_u32(smem + SMEM_Q), sP = smem_u32(smem + SMEM_P);
      bool ok = mbar_wait(q_full, 0, p.status, kStatusTimeoutMma);
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait(p_full, static_cast<uint32_t>(i & 1), p.status, kStatusTimeoutMma)) return false;
        const int st = i % VS;
        if (!mbar_wait(&v_full[st], static_cast<uint32_t>((i / VS) & 1), p.status, kStatusTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t sV = smem_u32(smem + SMEM_V + st * Cfg::V_BYTES);
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
        const int sb = j & 1, st = j % KS;  // S buffer, K stage
        if (!mbar_wait(&k_full[st], static_cast<uint32_t>((j / KS) & 1), p.status, kStatusTimeoutMma)) break;
        if (!mbar_wait(&s_free[sb], static_cast<uint32_t>(((j >> 1) & 1) ^ 1), p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        const uint32_t sK = smem_u32(smem + SMEM_K + st * Cfg::Q_BYTES);
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk) {
          const uint32_t off = (kk >> 2) * BOX_BYTES + (kk & 3) * 32;
          umma_f16_ss(tmem_base + TMEM_S0 + sb * BN, make_smem_desc_sw128(sQ + off, 16, 1024),
                      make_smem_desc_sw128(sK + off, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
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
        for (int c = 0; c < DV / 32; ++c) {
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
      __nv_bfloat16* og = p.o + ((static_cast<int64_t>(b) * p.S + (valid ? row : 0)) * p.Hq + h) * DV;
#pragma unroll
      for (int c = 0; c < DV / 32; ++c) {
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

template <int DQK, int DV, int KS, int VS>
static void launch_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, AttnTcParams& p, int dev) {
  using namespace attn_tc;
  using Cfg = FwdCfg<DQK, DV, KS, VS>;
  TmaSlots& ts = tls_tma_slots();
  const int box[4] = {64, BM, 1, 1};
  auto map = [&](CUtensorMap* m, const at::Tensor& t, int d) {
    const int64_t dims[4] = {d, t.size(1), t.size(2), t.size(0)};
    const int64_t str[3] = {t.stride(1), t.stride(2), t.stride(0)};
    make_tma_4d_bf16(m, t.data_ptr(), dims, str, box);
  };
  map(&ts.m[0], q, DQK);
  map(&ts.m[1], k, DQK);
  map(&ts.m[2], v, DV);
  auto kern = flash_fwd_tc_kernel<DQK, DV, KS, VS>;
  static bool attr_done[64] = {};
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    NTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    attr_done[dev] = true;
  }
  dim3 grid(static_cast<unsigned>((p.S + BM - 1) / BM), static_cast<unsigned>(p.Hq), static_cast<unsigned>(p.B));
  void* args[4] = {&ts.m[0], &ts.m[1], &ts.m[2], &p};
  NTB_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(kern), grid, dim3(192), args,
                                  static_cast<size_t>(Cfg::SMEM_BYTES), at::cuda::getCurrentCUDAStream(dev)));
  NTB_LAUNCH_CHECK(1);
}

bool flash_attn_fwd_tc_supported(int64_t dqk, int64_t dv) {
  return (dqk == 128 && dv == 128) || (dqk == 192 && dv == 128) || (dqk == 64 && dv == 64);
}

// q, k: [B, S, H, DQK], v: [B, S, Hkv, DV] bf16 views (head dim contiguous, 16-byte aligned strides);
// (DQK, DV) in {(128, 128), (192, 128) (MLA: [nope 128 | rope 64] x v 128), (64, 64)}.
std::vector<at::Tensor> flash_attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                                          bool causal) {
  using namespace attn_tc;
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "flash_attn_fwd_tc: [B, S, H, D] tensors");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "flash_attn_fwd_tc: bf16");
  const int64_t DQK = q.size(3), DV = v.size(3);
  TORCH_CHECK(k.size(3) == DQK && flash_attn_fwd_tc_supported(DQK, DV),
              "flash_attn_fwd_tc: head dims (q/k, v) must be (128, 128), (192, 128) or (64, 64)");
  TORCH_CHECK(q.stride(3) == 1 && k.stride(3) == 1 && v.stride(3) == 1, "flash_attn_fwd_tc: head dim contiguous");
  TORCH_CHECK(k.size(1) == q.size(1) && v.size(1) == q.size(1) && k.size(0) == q.size(0) && v.size(0) == q.size(0),
              "flash_attn_fwd_tc: self-attention shapes");
  TORCH_CHECK(q.size(2) % k.size(2) == 0 && k.size(2) == v.size(2), "flash_attn_fwd_tc: GQA head ratio");
  const int64_t B = q.size(0), S = q.size(1), Hq = q.size(2), Hkv = k.size(2);
  auto o = at::empty({B, S, Hq, DV}, q.options());
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
  if (DQK == 128) launch_fwd_tc<128, 128, 2, 2>(q, k, v, p, dev);
  else if (DQK == 192) launch_fwd_tc<192, 128, 1, 2>(q, k, v, p, dev);
  else launch_fwd_tc<64, 64, 2, 2>(q, k, v, p, dev);
  return {o, lse};
}


// ================================================================== backward
// One CTA per (128-key block, query head, batch), 192 threads; the CTA loops over the
// query blocks at or after the key block (causal) and accumulates its query head's
// share of dK and dV in TMEM (for GQA the shares of the heads of one group are then
// added with vector reductions into fp32 accumulators and converted to bf16):
//   per query block i:  S^T = K Q_i^T   (TMEM cols   0..127, lanes = keys)
//                       dP^T = V dO_i^T (TMEM cols 128..255)
//   threads (one per key row): P^T = 2^(S^T * scale_log2 - lse) -> smem (bf16)
//                       dV += P^T dO_i  (cols 384..511)
//   threads: dS^T = P^T (dP^T - delta) -> smem (bf16)
//                       dK += dS^T Q_i  (cols 256..383)
//                       dQ_i = dS K     (cols 0..127, lanes = queries; A = dS^T read MN-major)
//   threads (one per query row): dQ_i added into the fp32 accumulator with vector
//   reductions (the softmax scale is applied when it is converted to bf16).
// Shared memory: K, V resident (32 KB each), Q_i, dO_i (32 KB each), P^T, dS^T
// (32 KB each); every tile is two 16 KB [128 x 64] boxes with 128-byte swizzle.
namespace attn_tc_bwd {
constexpr int BM = 128, BN = 128;
constexpr int BOX = BM * 64 * 2;  // one [128 x 64] swizzled box, 16 KB
constexpr int PT = 2 * BOX;       // P^T / dS^T tile: 128 keys x 128 queries
constexpr uint32_t TMEM_COLS = 512;

// Plan of the backward for head dims DQK (q, k) and DV (v, o). SERIAL = false (DQK <= 128): S^T and
// dP^T get their own TMEM columns and are issued together; dQ reuses S^T's columns. SERIAL = true
// (MLA, DQK = 192): the TMEM cannot hold S^T, dP^T, dK (192) and dV at once, so dP^T is computed
// into S^T's columns after P^T was read out, and dQ (192 columns) overlaps them and the free tail;
// P^T and dS^T share one shared-memory tile (dS^T is written once dP^T, and with it the dV MMA
// that read P^T, completed).
template <int DQK, int DV, bool SERIAL>
struct BwdCfg {
  static_assert(DQK % 64 == 0 && DV % 64 == 0, "head dims");
  static constexpr int QB = DQK / 64, VB = DV / 64;
  static constexpr int Q_BYTES = QB * BOX, V_BYTES = VB * BOX;
  static constexpr int S_K = 0, S_V = S_K + Q_BYTES, S_Q = S_V + V_BYTES, S_DO = S_Q + Q_BYTES, S_P = S_DO + V_BYTES;
  static constexpr int S_DS = SERIAL ? S_P : S_P + PT;
  static constexpr int S_LSE = S_DS + PT;  // float[2][128] lse, float[2][128] delta (by iteration parity)
  static constexpr int S_BAR = S_LSE + 4 * 128 * 4;
  static constexpr int SMEM_BYTES = 1024 + S_BAR + 256;
  static constexpr uint32_t COL_S = SERIAL ? DQK + DV : 0;
  static constexpr uint32_t COL_DP = SERIAL ? COL_S : 128;
  static constexpr uint32_t COL_DK = SERIAL ? 0 : 256;
  static constexpr uint32_t COL_DV = COL_DK + DQK;
  static_assert(SMEM_BYTES <= 232448, "shared memory");
  static_assert(COL_S + DQK <= TMEM_COLS && COL_DV + DV <= TMEM_COLS && (SERIAL || COL_DV + DV <= 512),
                "TMEM columns");
  static_assert(SERIAL || DQK <= 128, "dQ reuses the 128 columns of S^T");
};
}  // namespace attn_tc_bwd

struct AttnTcBwdParams {
  const float* lse;    // [B, Hq, S] (log2 domain)
  const float* delta;  // [B, Hq, S]
  float* dq_acc;       // [B, Hq, S, D] fp32, unscaled dS K
  __nv_bfloat16* dk;   // strided [B, S, Hkv, D]
  __nv_bfloat16* dv;
  float* dk_acc;       // GQA or split: fp32 [B, S, Hkv, D] accumulators (every contributing CTA adds into them)
  float* dv_acc;
  int64_t dk_sb, dk_ss, dk_sh, dv_sb, dv_ss, dv_sh;
  int B, S, Hq, Hkv;
  float scale, scale_log2;
  int causal;
  int* status;
  // Serial kernel only: 0, or the most query blocks one CTA processes. With a split, blockIdx.x
  // enumerates (key block, run of at most qsplit query blocks) pairs, heaviest key blocks first,
  // and dK / dV always go through the fp32 accumulators.
  int qsplit;
};

// Key block and query-block run of this CTA (see AttnTcBwdParams::qsplit).
__device__ __forceinline__ void bwd_work_item(const AttnTcBwdParams& p, int nqb, int& kb, int& qb_first, int& iters) {
  if (p.qsplit <= 0) {
    kb = static_cast<int>(blockIdx.x);
    qb_first = p.causal ? kb : 0;
    iters = nqb - qb_first;
    return;
  }
  int rem = static_cast<int>(blockIdx.x);
  for (kb = 0; kb < nqb; ++kb) {
    const int first = p.causal ? kb : 0;
    const int cnt = nqb - first;
    const int runs = (cnt + p.qsplit - 1) / p.qsplit;
    if (rem < runs) {
      qb_first = first + rem * p.qsplit;
      iters = min(p.qsplit, cnt - rem * p.qsplit);
      return;
    }
    rem -= runs;
  }
  kb = 0;  // past the last item (the host sizes the grid exactly): no work
  qb_first = 0;
  iters = 0;
}

template <int DQK, int DV, bool SERIAL>
__global__ void __launch_bounds__(192, 1)
    flash_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        AttnTcBwdParams p) {
  using namespace attn_tc_bwd;
  using Cfg = BwdCfg<DQK, DV, SERIAL>;
  constexpr int S_K = Cfg::S_K, S_V = Cfg::S_V, S_Q = Cfg::S_Q, S_DO = Cfg::S_DO, S_P = Cfg::S_P, S_DS = Cfg::S_DS,
                S_LSE = Cfg::S_LSE, S_BAR = Cfg::S_BAR;
  constexpr uint32_t COL_S = Cfg::COL_S, COL_DP = Cfg::COL_DP, COL_DK = Cfg::COL_DK, COL_DV = Cfg::COL_DV;
  using attn_tc::ex2_approx;
  using attn_tc::warp_wait;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;
  uint64_t* do_full = bars + 2;
  uint64_t* q_free = bars + 3;
  uint64_t* do_free = bars + 4;
  uint64_t* s_full = bars + 5;   // S^T and dP^T ready
  uint64_t* p_ready = bars + 6;  // P^T in smem (128 arrivals)
  uint64_t* ds_ready = bars + 7; // dS^T in smem (128 arrivals)
  uint64_t* dq_full = bars + 8;
  uint64_t* dq_free = bars + 9;  // dQ read back (128 arrivals)
  uint64_t* kv_done = bars + 10;
  uint64_t* stats_ready = bars + 11;  // lse/delta of the iteration written (128 arrivals)
  uint64_t* dp_full = bars + 12;      // SERIAL: dP^T (and the dV MMA before it) complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  float* s_lse_all = reinterpret_cast<float*>(smem + S_LSE);  // [2][128]
  float* s_delta_all = s_lse_all + 256;                        // [2][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = blockIdx.y, b = blockIdx.z;
  const int group = p.Hq / p.Hkv;
  const int hk = hq / group;
  const int nqb = (p.S + BM - 1) / BM;
  int kb, qb_first, iters;  // heaviest (lowest) key blocks first
  bwd_work_item(p, nqb, kb, qb_first, iters);
  const int k0 = kb * BN;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(q_full, 1);
    mbar_init(do_full, 1);
    mbar_init(q_free, 1);
    mbar_init(do_free, 1);
    mbar_init(s_full, 1);
    mbar_init(p_ready, 128);
    mbar_init(ds_ready, 128);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 128);
    mbar_init(kv_done, 1);
    mbar_init(stats_ready, 128);
    mbar_init(dp_full, 1);
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
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
      mbar_expect_tx(kv_full, Cfg::Q_BYTES + Cfg::V_BYTES);
      for (int c = 0; c < Cfg::QB; ++c) tma_load_4d(smem + S_K + c * BOX, &tmK, kv_full, c * 64, k0, hk, b);
      for (int c = 0; c < Cfg::VB; ++c) tma_load_4d(smem + S_V + c * BOX, &tmV, kv_full, c * 64, k0, hk, b);
      for (int it = 0; it < iters; ++it) {
        const int h = hq;
        const int q0 = (qb_first + it) * BM;
        const uint32_t par = static_cast<uint32_t>(it & 1);
        if (!mbar_wait(q_free, par ^ 1, p.status, kStatusTimeoutProducer)) break;
        mbar_expect_tx(q_full, Cfg::Q_BYTES);
        for (int c = 0; c < Cfg::QB; ++c) tma_load_4d(smem + S_Q + c * BOX, &tmQ, q_full, c * 64, q0, h, b);
        if (!mbar_wait(do_free, par ^ 1, p.status, kStatusTimeoutProducer)) break;
        mbar_expect_tx(do_full, Cfg::V_BYTES);
        for (int c = 0; c < Cfg::VB; ++c) tma_load_4d(smem + S_DO + c * BOX, &tmDO, do_full, c * 64, q0, h, b);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_KK = make_idesc_f16(BM, BN, false, false);   // S^T, dP^T: both operands K-major (K = d)
      constexpr uint32_t ID_DV = make_idesc_f16(BM, DV, false, true);    // dV: A K-major (K = q), B N-major
      constexpr uint32_t ID_DK = make_idesc_f16(BM, DQK, false, true);   // dK: A K-major (K = q), B N-major
      constexpr uint32_t ID_NN = make_idesc_f16(BM, DQK, true, true);    // dQ: A M-major (dS^T), B N-major (K)
      const uint32_t sK = smem_u32(smem + S_K), sV = smem_u32(smem + S_V), sQ = smem_u32(smem + S_Q),
                     sDO = smem_u32(smem + S_DO), sP = smem_u32(smem + S_P), sDS = smem_u32(smem + S_DS);
      auto kdesc = [](uint32_t base, int kk) {  // K-major, K chunks of 64 in 16 KB boxes
        return make_smem_desc_sw128(base + (kk >> 2) * BOX + (kk & 3) * 32, 16, 1024);
      };
      auto ndesc = [](uint32_t base, int kk) {  // MN-major: 64-wide MN chunks 16 KB apart, k16 = 16 rows
        return make_smem_desc_sw128(base + kk * 2048, BOX, 1024);
      };
      bool ok = mbar_wait(kv_full, 0, p.status, kStatusTimeoutMma);
      for (int it = 0; ok && it < iters; ++it) {
        const uint32_t par = static_cast<uint32_t>(it & 1);
        if (!mbar_wait(q_full, par, p.status, kStatusTimeoutMma) ||
            !mbar_wait(do_full, par, p.status, kStatusTimeoutMma) ||
            !mbar_wait(dq_free, par ^ 1, p.status, kStatusTimeoutMma))
          break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk)
          umma_f16_ss(tmem_base + COL_S, kdesc(sK, kk), kdesc(sQ, kk), ID_KK, kk > 0 ? 1u : 0u);
        if (!SERIAL) {
#pragma unroll
          for (int kk = 0; kk < DV / 16; ++kk)
            umma_f16_ss(tmem_base + COL_DP, kdesc(sV, kk), kdesc(sDO, kk), ID_KK, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        if (!mbar_wait(p_ready, par, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        if (SERIAL) {  // S^T has been read out: dP^T into its columns
#pragma unroll
          for (int kk = 0; kk < DV / 16; ++kk)
            umma_f16_ss(tmem_base + COL_DP, kdesc(sV, kk), kdesc(sDO, kk), ID_KK, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk)
          umma_f16_ss(tmem_base + COL_DV, kdesc(sP, kk), ndesc(sDO, kk), ID_DV, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(do_free);
        if (SERIAL) umma_commit(dp_full);
        if (!mbar_wait(ds_ready, par, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk)
          umma_f16_ss(tmem_base + COL_DK, kdesc(sDS, kk), ndesc(sQ, kk), ID_DK, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(q_free);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_f16_ss(tmem_base + COL_S, ndesc(sDS, kk), ndesc(sK, kk), ID_NN, kk > 0 ? 1u : 0u);
        umma_commit(dq_full);
      }
      umma_commit(kv_done);
      mbar_wait(kv_done, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ compute warps
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row for S^T/dP^T/dK/dV; query row for dQ
    const int key = k0 + r;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int ctid = threadIdx.x - 64;
    uint8_t* sP = smem + S_P;
    uint8_t* sDS = smem + S_DS;
    bool ok = true;
    // lse / delta of one query block (+inf / 0 beyond S: P = 0 there); the next block's values
    // are loaded one iteration ahead so the global-memory latency is off the critical path.
    auto load_stats = [&](int itx, float& lv, float& dv) {
      const int hx = hq;
      const int qx = (qb_first + itx) * BM + ctid;
      const int64_t o = (static_cast<int64_t>(b) * p.Hq + hx) * p.S + qx;
      lv = qx < p.S ? p.lse[o] : INFINITY;
      dv = qx < p.S ? p.delta[o] : 0.f;
    };
    float next_lse = 0.f, next_delta = 0.f;
    if (iters > 0) load_stats(0, next_lse, next_delta);
    for (int it = 0; it < iters; ++it) {
      const int h = hq;
      const int q0 = (qb_first + it) * BM;
      const uint32_t par = static_cast<uint32_t>(it & 1);
      // Double-buffered by iteration parity: a thread writes buffer it & 1 only after every
      // compute thread arrived for iteration it - 1, i.e. finished with iteration it - 2's buffer.
      float* s_lse = s_lse_all + (it & 1) * 128;
      float* s_delta = s_delta_all + (it & 1) * 128;
      s_lse[ctid] = next_lse;
      s_delta[ctid] = next_delta;
      if (it + 1 < iters) load_stats(it + 1, next_lse, next_delta);
      mbar_arrive(stats_ready);
      if (!warp_wait(stats_ready, par, p.status, kStatusTimeoutEpilogue) ||
          !warp_wait(s_full, par, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = p.causal && q0 == k0;
      const bool row_dead = key >= p.S;
      // P^T row (keys x queries): kept packed in registers for dS, stored to smem for dV.
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t sr[32];
        tmem_ld32(tmem_base + lane_addr + COL_S + c * 32, sr);
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const int qa = c * 32 + t;
          float e0 = ex2_approx(fmaf(__uint_as_float(sr[t]), p.scale_log2, -s_lse[qa]));
          float e1 = ex2_approx(fmaf(__uint_as_float(sr[t + 1]), p.scale_log2, -s_lse[qa + 1]));
          if (row_dead || (diag && r > qa)) e0 = 0.f;
          if (row_dead || (diag && r > qa + 1)) e1 = 0.f;
          pk[(c * 32 + t) >> 1] = pack_bf16x2(e0, e1);
        }
      }
#pragma unroll
      for (int c16 = 0; c16 < 16; ++c16) {
        const uint4 v = make_uint4(pk[c16 * 4], pk[c16 * 4 + 1], pk[c16 * 4 + 2], pk[c16 * 4 + 3]);
        *reinterpret_cast<uint4*>(sP + (c16 >> 3) * BOX + r * 128 + (((c16 & 7) ^ (r & 7)) << 4)) = v;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(p_ready);
      if (SERIAL) {  // dP^T lands in S^T's columns; the dV MMA reading P^T completed before it
        if (!warp_wait(dp_full, par, p.status, kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // dS^T = P^T * (dP^T - delta)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t dr[32];
        tmem_ld32(tmem_base + lane_addr + COL_DP + c * 32, dr);
        uint32_t ds[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const int qa = c * 32 + t;
          const uint32_t pp = pk[qa >> 1];
          const float d0 = bf16_lo(pp) * (__uint_as_float(dr[t]) - s_delta[qa]);
          const float d1 = bf16_hi(pp) * (__uint_as_float(dr[t + 1]) - s_delta[qa + 1]);
          ds[t >> 1] = pack_bf16x2(d0, d1);
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int c16 = c * 4 + q4;
          const uint4 v = make_uint4(ds[q4 * 4], ds[q4 * 4 + 1], ds[q4 * 4 + 2], ds[q4 * 4 + 3]);
          *reinterpret_cast<uint4*>(sDS + (c16 >> 3) * BOX + r * 128 + (((c16 & 7) ^ (r & 7)) << 4)) = v;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(ds_ready);
      // dQ_i (lanes = queries) -> fp32 accumulator.
      if (!warp_wait(dq_full, par, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int q = q0 + r;
      float* dst = p.dq_acc + ((static_cast<int64_t>(b) * p.Hq + h) * p.S + (q < p.S ? q : 0)) * DQK;
#pragma unroll
      for (int c = 0; c < DQK / 32; ++c) {
        uint32_t qr[32];
        tmem_ld32(tmem_base + lane_addr + COL_S + c * 32, qr);
        if (q < p.S) {
#pragma unroll
          for (int t = 0; t < 32; t += 4)
            red_add_v4(dst + c * 32 + t, __uint_as_float(qr[t]), __uint_as_float(qr[t + 1]),
                       __uint_as_float(qr[t + 2]), __uint_as_float(qr[t + 3]));
        }
      }
      tc_fence_before();
      mbar_arrive(dq_free);
    }
    // dK (scaled) and dV rows of this key block: stored directly (one query head per kv head)
    // or added into the fp32 accumulators (GQA).
    if (ok && warp_wait(kv_done, 0, p.status, kStatusTimeoutEpilogue)) {
      tc_fence_after();
      const bool valid = key < p.S;
      const int64_t krow = valid ? key : 0;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const uint32_t col = which == 0 ? COL_DK : COL_DV;
        const int width = which == 0 ? DQK : DV;
        const float sc = which == 0 ? p.scale : 1.f;
        float* accp = which == 0 ? p.dk_acc : p.dv_acc;
        __nv_bfloat16* out = which == 0 ? p.dk + b * p.dk_sb + krow * p.dk_ss + hk * p.dk_sh
                                        : p.dv + b * p.dv_sb + krow * p.dv_ss + hk * p.dv_sh;
        float* acc_row =
            accp != nullptr ? accp + ((static_cast<int64_t>(b) * p.S + krow) * p.Hkv + hk) * width : nullptr;
#pragma unroll 1
        for (int c = 0; c < width / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem_base + lane_addr + col + c * 32, v);
          if (!valid) continue;
          if (acc_row != nullptr) {
#pragma unroll
            for (int t = 0; t < 32; t += 4)
              red_add_v4(acc_row + c * 32 + t, __uint_as_float(v[t]) * sc, __uint_as_float(v[t + 1]) * sc,
                         __uint_as_float(v[t + 2]) * sc, __uint_as_float(v[t + 3]) * sc);
          } else {
#pragma unroll
            for (int t = 0; t < 32; t += 8) {
              uint4 o;
              o.x = pack_bf16x2(__uint_as_float(v[t]) * sc, __uint_as_float(v[t + 1]) * sc);
              o.y = pack_bf16x2(__uint_as_float(v[t + 2]) * sc, __uint_as_float(v[t + 3]) * sc);
              o.z = pack_bf16x2(__uint_as_float(v[t + 4]) * sc, __uint_as_float(v[t + 5]) * sc);
              o.w = pack_bf16x2(__uint_as_float(v[t + 6]) * sc, __uint_as_float(v[t + 7]) * sc);
              *reinterpret_cast<uint4*>(out + c * 32 + t) = o;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, attn_tc_bwd::TMEM_COLS);
  }
}

// Pipelined backward for head dims <= 128 (flash_bwd_tc_pipe_kernel). Same math and outputs as
// flash_bwd_tc_kernel, with a schedule that keeps the tensor core fed across query blocks:
//   * Q is double-buffered in shared memory (Q(i+1) is loaded while block i is processed); P^T and
//     dS^T share one tile (dS^T is stored once the dV MMA that reads P^T has completed);
//   * dQ is computed into dP^T's TMEM columns, so S^T(i+1) = K Q(i+1)^T is issued right after the
//     dK / dQ MMAs of block i and runs while the threads drain dQ(i) into the fp32 accumulator;
//     dP^T(i+1) follows once that readout is done.
// TMEM: S^T [0, 128), dP^T / dQ [128, 256), dK [256, 256 + DQK), dV [256 + DQK, ... + DV).
namespace attn_tc_bwd {
template <int DQK, int DV>
struct BwdPipeCfg {
  static_assert(DQK % 64 == 0 && DV % 64 == 0 && DQK <= 128 && DV <= 128, "head dims");
  static constexpr int QB = DQK / 64, VB = DV / 64;
  static constexpr int Q_BYTES = QB * BOX, V_BYTES = VB * BOX;
  static constexpr int S_K = 0, S_V = S_K + Q_BYTES, S_Q = S_V + V_BYTES, S_DO = S_Q + 2 * Q_BYTES;
  static constexpr int S_P = S_DO + V_BYTES;  // P^T, then dS^T
  static constexpr int S_LSE = S_P + PT;
  static constexpr int S_BAR = S_LSE + 4 * 128 * 4;
  static constexpr int SMEM_BYTES = 1024 + S_BAR + 256;
  static constexpr uint32_t COL_S = 0, COL_DP = 128, COL_DK = 256, COL_DV = 256 + DQK;
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};
}  // namespace attn_tc_bwd

template <int DQK, int DV>
__global__ void __launch_bounds__(192, 1)
    flash_bwd_tc_pipe_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                             AttnTcBwdParams p) {
  using namespace attn_tc_bwd;
  using attn_tc::ex2_approx;
  using attn_tc::warp_wait;
  using Cfg = BwdPipeCfg<DQK, DV>;
  constexpr int S_K = Cfg::S_K, S_V = Cfg::S_V, S_Q = Cfg::S_Q, S_DO = Cfg::S_DO, S_P = Cfg::S_P,
                S_LSE = Cfg::S_LSE, S_BAR = Cfg::S_BAR;
  constexpr uint32_t COL_S = Cfg::COL_S, COL_DP = Cfg::COL_DP, COL_DK = Cfg::COL_DK, COL_DV = Cfg::COL_DV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;       // [2]
  uint64_t* q_free = bars + 3;       // [2] dK of the block in this slot completed
  uint64_t* do_full = bars + 5;
  uint64_t* do_free = bars + 6;      // dP^T and dV of the block completed
  uint64_t* s_full = bars + 7;       // S^T ready
  uint64_t* dp_full = bars + 8;      // dP^T ready
  uint64_t* p_ready = bars + 9;      // P^T in smem, S^T read (128 arrivals)
  uint64_t* dv_done = bars + 10;     // dV MMA completed: the P^T tile may be overwritten
  uint64_t* ds_ready = bars + 11;    // dS^T in smem, dP^T read (128 arrivals)
  uint64_t* dq_full = bars + 12;     // dK and dQ MMAs completed
  uint64_t* dq_free = bars + 13;     // dQ read out of TMEM (128 arrivals)
  uint64_t* kv_done = bars + 14;
  uint64_t* stats_ready = bars + 15; // lse/delta of the iteration written (128 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  float* s_lse_all = reinterpret_cast<float*>(smem + S_LSE);  // [2][128]
  float* s_delta_all = s_lse_all + 256;                        // [2][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = blockIdx.x;
  const int hq = blockIdx.y, b = blockIdx.z;
  const int hk = hq / (p.Hq / p.Hkv);
  const int k0 = kb * BN;
  const int nqb = (p.S + BM - 1) / BM;
  const int qb_first = p.causal ? kb : 0;
  const int iters = nqb - qb_first;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_free[i], 1);
    }
    mbar_init(do_full, 1);
    mbar_init(do_free, 1);
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 128);
    mbar_init(dv_done, 1);
    mbar_init(ds_ready, 128);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 128);
    mbar_init(kv_done, 1);
    mbar_init(stats_ready, 128);
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
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
      mbar_expect_tx(kv_full, Cfg::Q_BYTES + Cfg::V_BYTES);
      for (int c = 0; c < Cfg::QB; ++c) tma_load_4d(smem + S_K + c * BOX, &tmK, kv_full, c * 64, k0, hk, b);
      for (int c = 0; c < Cfg::VB; ++c) tma_load_4d(smem + S_V + c * BOX, &tmV, kv_full, c * 64, k0, hk, b);
      for (int it = 0; it < iters; ++it) {
        const int q0 = (qb_first + it) * BM;
        const int qs = it & 1;
        if (!mbar_wait(&q_free[qs], static_cast<uint32_t>((it >> 1) & 1) ^ 1u, p.status, kStatusTimeoutProducer))
          break;
        mbar_expect_tx(&q_full[qs], Cfg::Q_BYTES);
        for (int c = 0; c < Cfg::QB; ++c)
          tma_load_4d(smem + S_Q + qs * Cfg::Q_BYTES + c * BOX, &tmQ, &q_full[qs], c * 64, q0, hq, b);
        if (!mbar_wait(do_free, static_cast<uint32_t>(it & 1) ^ 1u, p.status, kStatusTimeoutProducer)) break;
        mbar_expect_tx(do_full, Cfg::V_BYTES);
        for (int c = 0; c < Cfg::VB; ++c) tma_load_4d(smem + S_DO + c * BOX, &tmDO, do_full, c * 64, q0, hq, b);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_KK = make_idesc_f16(BM, BN, false, false);
      constexpr uint32_t ID_DV = make_idesc_f16(BM, DV, false, true);
      constexpr uint32_t ID_DK = make_idesc_f16(BM, DQK, false, true);
      constexpr uint32_t ID_NN = make_idesc_f16(BM, DQK, true, true);
      const uint32_t sK = smem_u32(smem + S_K), sV = smem_u32(smem + S_V), sDO = smem_u32(smem + S_DO),
                     sP = smem_u32(smem + S_P);
      auto kdesc = [](uint32_t base, int kk) { return make_smem_desc_sw128(base + (kk >> 2) * BOX + (kk & 3) * 32, 16, 1024); };
      auto ndesc = [](uint32_t base, int kk) { return make_smem_desc_sw128(base + kk * 2048, BOX, 1024); };
      auto sq = [&](int it) { return smem_u32(smem + S_Q + (it & 1) * Cfg::Q_BYTES); };
      auto issue_s = [&](int it) {
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk)
          umma_f16_ss(tmem_base + COL_S, kdesc(sK, kk), kdesc(sq(it), kk), ID_KK, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
      };
      auto issue_dp = [&]() {
#pragma unroll
        for (int kk = 0; kk < DV / 16; ++kk)
          umma_f16_ss(tmem_base + COL_DP, kdesc(sV, kk), kdesc(sDO, kk), ID_KK, kk > 0 ? 1u : 0u);
        umma_commit(dp_full);
      };
      bool ok = mbar_wait(kv_full, 0, p.status, kStatusTimeoutMma) && iters > 0 &&
                mbar_wait(&q_full[0], 0, p.status, kStatusTimeoutMma) && mbar_wait(do_full, 0, p.status, kStatusTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        issue_dp();
      }
      for (int it = 0; ok && it < iters; ++it) {
        const uint32_t par = static_cast<uint32_t>(it & 1);
        if (!mbar_wait(p_ready, par, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk)
          umma_f16_ss(tmem_base + COL_DV, kdesc(sP, kk), ndesc(sDO, kk), ID_DV, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(do_free);
        umma_commit(dv_done);
        if (!mbar_wait(ds_ready, par, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk)
          umma_f16_ss(tmem_base + COL_DK, kdesc(sP, kk), ndesc(sq(it), kk), ID_DK, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&q_free[it & 1]);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_f16_ss(tmem_base + COL_DP, ndesc(sP, kk), ndesc(sK, kk), ID_NN, kk > 0 ? 1u : 0u);
        umma_commit(dq_full);
        if (it + 1 < iters) {
          const int nx = it + 1;
          if (!mbar_wait(&q_full[nx & 1], static_cast<uint32_t>((nx >> 1) & 1), p.status, kStatusTimeoutMma)) break;
          tc_fence_after();
          issue_s(nx);  // S^T(it) was read before p_ready(it)
          if (!mbar_wait(do_full, static_cast<uint32_t>(nx & 1), p.status, kStatusTimeoutMma) ||
              !mbar_wait(dq_free, par, p.status, kStatusTimeoutMma))
            break;
          tc_fence_after();
          issue_dp();  // dQ(it) has been read out of these columns
        }
      }
      umma_commit(kv_done);
      mbar_wait(kv_done, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ compute warps
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row for S^T/dP^T/dK/dV; query row for dQ
    const int key = k0 + r;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int ctid = threadIdx.x - 64;
    uint8_t* sP = smem + S_P;
    bool ok = true;
    auto load_stats = [&](int itx, float& lv, float& dv) {
      const int qx = (qb_first + itx) * BM + ctid;
      const int64_t o = (static_cast<int64_t>(b) * p.Hq + hq) * p.S + qx;
      lv = qx < p.S ? p.lse[o] : INFINITY;
      dv = qx < p.S ? p.delta[o] : 0.f;
    };
    float next_lse = 0.f, next_delta = 0.f;
    if (iters > 0) load_stats(0, next_lse, next_delta);
    for (int it = 0; it < iters; ++it) {
      const int q0 = (qb_first + it) * BM;
      const uint32_t par = static_cast<uint32_t>(it & 1);
      float* s_lse = s_lse_all + (it & 1) * 128;
      float* s_delta = s_delta_all + (it & 1) * 128;
      s_lse[ctid] = next_lse;
      s_delta[ctid] = next_delta;
      if (it + 1 < iters) load_stats(it + 1, next_lse, next_delta);
      mbar_arrive(stats_ready);
      if (!warp_wait(stats_ready, par, p.status, kStatusTimeoutEpilogue) ||
          !warp_wait(s_full, par, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = p.causal && q0 == k0;
      const bool row_dead = key >= p.S;
      // P^T row: packed bf16 in registers (for dS^T) and stored to the shared tile (for dV). The
      // tile held dS^T(it - 1), whose MMAs completed before dq_full(it - 1) was observed.
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t sr[32];
        tmem_ld32(tmem_base + lane_addr + COL_S + c * 32, sr);
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const int qa = c * 32 + t;
          float e0 = ex2_approx(fmaf(__uint_as_float(sr[t]), p.scale_log2, -s_lse[qa]));
          float e1 = ex2_approx(fmaf(__uint_as_float(sr[t + 1]), p.scale_log2, -s_lse[qa + 1]));
          if (row_dead || (diag && r > qa)) e0 = 0.f;
          if (row_dead || (diag && r > qa + 1)) e1 = 0.f;
          pk[(c * 32 + t) >> 1] = pack_bf16x2(e0, e1);
        }
      }
#pragma unroll
      for (int c16 = 0; c16 < 16; ++c16) {
        const uint4 v = make_uint4(pk[c16 * 4], pk[c16 * 4 + 1], pk[c16 * 4 + 2], pk[c16 * 4 + 3]);
        *reinterpret_cast<uint4*>(sP + (c16 >> 3) * BOX + r * 128 + (((c16 & 7) ^ (r & 7)) << 4)) = v;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(p_ready);
      // dS^T = P^T * (dP^T - delta), kept packed until the dV MMA has finished reading P^T.
      if (!warp_wait(dp_full, par, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t ds[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t dr[32];
        tmem_ld32(tmem_base + lane_addr + COL_DP + c * 32, dr);
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const int qa = c * 32 + t;
          const uint32_t pp = pk[qa >> 1];
          const float d0 = bf16_lo(pp) * (__uint_as_float(dr[t]) - s_delta[qa]);
          const float d1 = bf16_hi(pp) * (__uint_as_float(dr[t + 1]) - s_delta[qa + 1]);
          ds[qa >> 1] = pack_bf16x2(d0, d1);
        }
      }
      if (!warp_wait(dv_done, par, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c16 = 0; c16 < 16; ++c16) {
        const uint4 v = make_uint4(ds[c16 * 4], ds[c16 * 4 + 1], ds[c16 * 4 + 2], ds[c16 * 4 + 3]);
        *reinterpret_cast<uint4*>(sP + (c16 >> 3) * BOX + r * 128 + (((c16 & 7) ^ (r & 7)) << 4)) = v;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(ds_ready);
      // dQ(it) (lanes = queries) from dP^T's columns -> fp32 accumulator.
      if (!warp_wait(dq_full, par, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int q = q0 + r;
      float* dst = p.dq_acc + ((static_cast<int64_t>(b) * p.Hq + hq) * p.S + (q < p.S ? q : 0)) * DQK;
#pragma unroll
      for (int c = 0; c < DQK / 32; ++c) {
        uint32_t qr[32];
        tmem_ld32(tmem_base + lane_addr + COL_DP + c * 32, qr);
        if (q < p.S) {
#pragma unroll
          for (int t = 0; t < 32; t += 4)
            red_add_v4(dst + c * 32 + t, __uint_as_float(qr[t]), __uint_as_float(qr[t + 1]),
                       __uint_as_float(qr[t + 2]), __uint_as_float(qr[t + 3]));
        }
      }
      tc_fence_before();
      mbar_arrive(dq_free);
    }
    if (ok && warp_wait(kv_done, 0, p.status, kStatusTimeoutEpilogue)) {
      tc_fence_after();
      const bool valid = key < p.S;
      const int64_t krow = valid ? key : 0;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const uint32_t col = which == 0 ? COL_DK : COL_DV;
        const int width = which == 0 ? DQK : DV;
        const float sc = which == 0 ? p.scale : 1.f;
        float* accp = which == 0 ? p.dk_acc : p.dv_acc;
        __nv_bfloat16* out = which == 0 ? p.dk + b * p.dk_sb + krow * p.dk_ss + hk * p.dk_sh
                                        : p.dv + b * p.dv_sb + krow * p.dv_ss + hk * p.dv_sh;
        float* acc_row =
            accp != nullptr ? accp + ((static_cast<int64_t>(b) * p.S + krow) * p.Hkv + hk) * width : nullptr;
#pragma unroll 1
        for (int c = 0; c < width / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem_base + lane_addr + col + c * 32, v);
          if (!valid) continue;
          if (acc_row != nullptr) {
#pragma unroll
            for (int t = 0; t < 32; t += 4)
              red_add_v4(acc_row + c * 32 + t, __uint_as_float(v[t]) * sc, __uint_as_float(v[t + 1]) * sc,
                         __uint_as_float(v[t + 2]) * sc, __uint_as_float(v[t + 3]) * sc);
          } else {
#pragma unroll
            for (int t = 0; t < 32; t += 8) {
              uint4 o;
              o.x = pack_bf16x2(__uint_as_float(v[t]) * sc, __uint_as_float(v[t + 1]) * sc);
              o.y = pack_bf16x2(__uint_as_float(v[t + 2]) * sc, __uint_as_float(v[t + 3]) * sc);
              o.z = pack_bf16x2(__uint_as_float(v[t + 4]) * sc, __uint_as_float(v[t + 5]) * sc);
              o.w = pack_bf16x2(__uint_as_float(v[t + 6]) * sc, __uint_as_float(v[t + 7]) * sc);
              *reinterpret_cast<uint4*>(out + c * 32 + t) = o;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, attn_tc_bwd::TMEM_COLS);
  }
}

// fp32 [B, S, H, D] accumulator -> bf16 strided [B, S, H, D] view, 8 elements per thread (two
// 16-byte loads, one 16-byte store; D % 8 == 0 and 16-byte aligned output rows, else 4 with an
// 8-byte store).
template <int V>
__global__ void acc_to_bf16_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ out, int B, int S, int H,
                                   int D, int64_t sb, int64_t ss, int64_t sh) {
  const int64_t total = static_cast<int64_t>(B) * S * H * D / V;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i * V;
    const int d = static_cast<int>(e % D);
    const int64_t r = e / D;
    const int h = static_cast<int>(r % H);
    const int64_t bs = r / H;
    const int s = static_cast<int>(bs % S);
    const int bb = static_cast<int>(bs / S);
    __nv_bfloat16* o = out + bb * sb + s * ss + h * sh + d;
    const float4 v = *reinterpret_cast<const float4*>(acc + e);
    if constexpr (V == 8) {
      const float4 w = *reinterpret_cast<const float4*>(acc + e + 4);
      *reinterpret_cast<uint4*>(o) = make_uint4(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w), pack_bf16x2(w.x, w.y),
                                                pack_bf16x2(w.z, w.w));
    } else {
      *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
    }
  }
}

bool flash_attn_bwd_tc_supported(int64_t dqk, int64_t dv) {
  return (dqk == 128 && dv == 128) || (dqk == 192 && dv == 128) || (dqk == 64 && dv == 64);
}

template <int DQK, int DV, bool SERIAL, bool PIPE>
constexpr int bwd_smem_bytes() {
  if constexpr (PIPE) return attn_tc_bwd::BwdPipeCfg<DQK, DV>::SMEM_BYTES;
  else return attn_tc_bwd::BwdCfg<DQK, DV, SERIAL>::SMEM_BYTES;
}

template <int DQK, int DV, bool SERIAL, bool PIPE = false>
static void launch_bwd_tc(AttnTcBwdParams& p, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                          const at::Tensor& dout, int dev, cudaStream_t stream) {
  using namespace attn_tc_bwd;
  constexpr int SMEM = bwd_smem_bytes<DQK, DV, SERIAL, PIPE>();
  TmaSlots& ts = tls_tma_slots();
  const int box[4] = {64, BM, 1, 1};
  auto map = [&](CUtensorMap* m, const at::Tensor& t, int d) {
    const int64_t dims[4] = {d, t.size(1), t.size(2), t.size(0)};
    const int64_t str[3] = {t.stride(1), t.stride(2), t.stride(0)};
    make_tma_4d_bf16(m, t.data_ptr(), dims, str, box);
  };
  map(&ts.m[0], q, DQK);
  map(&ts.m[1], k, DQK);
  map(&ts.m[2], v, DV);
  map(&ts.m[3], dout, DV);
  void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, AttnTcBwdParams);
  if constexpr (PIPE) kern = flash_bwd_tc_pipe_kernel<DQK, DV>;
  else kern = flash_bwd_tc_kernel<DQK, DV, SERIAL>;
  static bool attr_done[64] = {};
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    NTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    attr_done[dev] = true;
  }
  const int nqb = (p.S + BN - 1) / BN;
  int items = nqb;
  if (!PIPE && p.qsplit > 0) {
    items = 0;
    for (int kb = 0; kb < nqb; ++kb) items += (nqb - (p.causal ? kb : 0) + p.qsplit - 1) / p.qsplit;
  }
  dim3 grid(static_cast<unsigned>(items), static_cast<unsigned>(p.Hq), static_cast<unsigned>(p.B));
  void* args[5] = {&ts.m[0], &ts.m[1], &ts.m[2], &ts.m[3], &p};
  NTB_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(kern), grid, dim3(192), args,
                                  static_cast<size_t>(SMEM), stream));
  NTB_LAUNCH_CHECK(1);
}

// Launches the tcgen05 backward for (q/k, v) head dims (128, 128), (192, 128) or (64, 64). dq_acc
// (fp32 [B, Hq, S, DQK]) must be zeroed; dk/dv are written in full (every key row of every kv head).
void flash_attn_bwd_tc_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
                              const at::Tensor& lse, const at::Tensor& delta, at::Tensor& dq_acc, at::Tensor& dk,
                              at::Tensor& dv, double scale, bool causal) {
  const int64_t DQK = q.size(3), DV = v.size(3);
  TORCH_CHECK(k.size(3) == DQK && flash_attn_bwd_tc_supported(DQK, DV), "flash_attn_bwd_tc: head dims");
  TORCH_CHECK(dout.is_contiguous() && dq_acc.is_contiguous(), "flash_attn_bwd_tc: contiguous dO and dq_acc");
  const int64_t B = q.size(0), S = q.size(1), Hq = q.size(2), Hkv = k.size(2);
  AttnTcBwdParams p{};
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.dk_sb = dk.stride(0); p.dk_ss = dk.stride(1); p.dk_sh = dk.stride(2);
  p.dv_sb = dv.stride(0); p.dv_ss = dv.stride(1); p.dv_sh = dv.stride(2);
  p.B = static_cast<int>(B);
  p.S = static_cast<int>(S);
  p.Hq = static_cast<int>(Hq);
  p.Hkv = static_cast<int>(Hkv);
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  const int dev = q.get_device();
  p.status = device_status(dev);
  at::Tensor dk_acc, dv_acc;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  // The pipelined variant (double-buffered Q, S of the next block issued under this block's
  // softmax) measured 1009 us against 941 us for the serial chain on the Llama shape (B=1,
  // S=4096, 32q/8kv heads, d=128, causal), so it runs only with NTB_ATTN_BWD_PIPE=1.
  const char* pipe_env = std::getenv("NTB_ATTN_BWD_PIPE");
  const bool pipe = pipe_env != nullptr && pipe_env[0] == '1' && DQK != 192;
  // Query-run split of the serial kernel: one CTA per (key block, query head) gives few, very
  // unequal CTAs when the heads per rank are few (tensor parallelism: 4 query heads at TP = 8 make
  // 128 CTAs on 148 SMs, the first key block running 32 query blocks and the last one). Runs of
  // at most qsplit query blocks, about two per SM, bound the longest CTA; dK / dV then add into
  // the fp32 accumulators. NTB_ATTN_BWD_SPLIT=0 turns it off.
  {
    const int64_t nqb = (S + 127) / 128;
    int64_t work = 0;
    for (int64_t kb = 0; kb < nqb; ++kb) work += nqb - (causal ? kb : 0);
    work *= Hq * B;
    const int64_t target = 2LL * num_sms(dev);
    const int64_t run = std::max<int64_t>(4, (work + target - 1) / target);
    const char* split_env = std::getenv("NTB_ATTN_BWD_SPLIT");
    const bool split_on = !(split_env != nullptr && split_env[0] == '0');
    p.qsplit = (!pipe && split_on && run < nqb) ? static_cast<int>(run) : 0;
  }
  if (Hq != Hkv || p.qsplit > 0) {
    dk_acc = at::zeros({B, S, Hkv, DQK}, q.options().dtype(at::kFloat));
    dv_acc = at::zeros({B, S, Hkv, DV}, q.options().dtype(at::kFloat));
    p.dk_acc = dk_acc.data_ptr<float>();
    p.dv_acc = dv_acc.data_ptr<float>();
  }
  if (DQK == 192) launch_bwd_tc<192, 128, true>(p, q, k, v, dout, dev, stream);
  else if (DQK == 128 && pipe) launch_bwd_tc<128, 128, false, true>(p, q, k, v, dout, dev, stream);
  else if (DQK == 128) launch_bwd_tc<128, 128, false>(p, q, k, v, dout, dev, stream);
  else if (pipe) launch_bwd_tc<64, 64, false, true>(p, q, k, v, dout, dev, stream);
  else launch_bwd_tc<64, 64, false>(p, q, k, v, dout, dev, stream);
  if (Hq != Hkv || p.qsplit > 0) {
    TORCH_CHECK(dk.stride(3) == 1 && dv.stride(3) == 1 && dk.stride(2) % 4 == 0 && dk.stride(1) % 4 == 0 &&
                    dv.stride(2) % 4 == 0 && dv.stride(1) % 4 == 0,
                "flash_attn_bwd_tc: dk/dv strides must keep 8-byte alignment");
    auto convert = [&](const at::Tensor& acc, __nv_bfloat16* o, int64_t D, int64_t sb, int64_t ss, int64_t sh) {
      const bool v8 = D % 8 == 0 && sb % 8 == 0 && ss % 8 == 0 && sh % 8 == 0 &&
                      (reinterpret_cast<uintptr_t>(o) & 15) == 0;
      const int64_t n = B * S * Hkv * D / (v8 ? 8 : 4);
      const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 8));
      if (v8)
        acc_to_bf16_kernel<8><<<blocks, 256, 0, stream>>>(acc.data_ptr<float>(), o, p.B, p.S, p.Hkv,
                                                          static_cast<int>(D), sb, ss, sh);
      else
        acc_to_bf16_kernel<4><<<blocks, 256, 0, stream>>>(acc.data_ptr<float>(), o, p.B, p.S, p.Hkv,
                                                          static_cast<int>(D), sb, ss, sh);
    };
    convert(dk_acc, p.dk, DQK, p.dk_sb, p.dk_ss, p.dk_sh);
    convert(dv_acc, p.dv, DV, p.dv_sb, p.dv_ss, p.dv_sh);
    NTB_LAUNCH_CHECK(2);
  }
}

}  // namespace ntb
