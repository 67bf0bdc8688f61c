// Causal flash attention, forward and backward, for sm_100a.
//
// Layouts: q [B,S,Hq,Dqk], k [B,S,Hkv,Dqk], v [B,S,Hkv,Dv] given by strides
// (views into a fused QKV projection output need no copy); o [B,S,Hq,Dv]
// contiguous; lse [B,Hq,S] fp32 in the log2 domain (log2 of the softmax
// denominator of scores scaled by softmax_scale*log2(e)).
//
// Forward: one CTA per (128-query block, head, batch), 8 warps x 16 rows,
// K/V blocks of 64 keys double-buffered with cp.async, online softmax in
// registers, P re-used from the S accumulators as the A operand of P.V.
// Backward: one CTA per (128-key block, kv head, batch), 8 warps x 16 keys,
// looping over the query heads of the GQA group and the query blocks at or
// below the diagonal; dK/dV stay in registers, dQ partial tiles are staged in
// shared memory and added to an fp32 accumulator with one bulk-async
// reduction (cp.reduce.async.bulk ... add.f32) per tile instead of
// per-element atomics.
//
// Reference parity: src/models/deepseek.py:681-738 (MLA, materialised scores,
// fp32 softmax), src/models/attention.py:134-220 (MHA). GQA (the reference
// never uses num_key_value_heads) is a B200-build extension needed by the
// Llama-shape benchmark.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include <cstdlib>

#include "common.cuh"
#include "host_utils.h"

namespace ntb {

using bf16 = __nv_bfloat16;

// tcgen05 backward for head dim 128 (attention_tc.cu).
void flash_attn_bwd_tc_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
                              const at::Tensor& lse, const at::Tensor& delta, at::Tensor& dq_acc, at::Tensor& dk,
                              at::Tensor& dv, double scale, bool causal);
bool flash_attn_bwd_tc_supported(int64_t dqk, int64_t dv);

// ---------------------------------------------------------------- helpers
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(g), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset of element (row, col) in a [rows][D] bf16 tile whose 16-byte
// chunks are XOR-swizzled with the row index (conflict-free ldmatrix).
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int col) {
  constexpr int CH = D / 8;
  constexpr int MASK = CH >= 8 ? 7 : CH - 1;
  return static_cast<uint32_t>(row * (D * 2) + ((((col >> 3) ^ (row & MASK))) << 4) + ((col & 7) << 1));
}

template <int ROWS, int D, int NT>
__device__ __forceinline__ void load_tile(bf16* s, const bf16* g, int64_t row_stride, int row0, int nrows, int tid) {
  constexpr int CH = D / 8;
  const uint32_t sb = smem_u32(s);
#pragma unroll 4
  for (int i = tid; i < ROWS * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    const int gr = row0 + r;
    const bool valid = gr < nrows;
    const bf16* src = g + static_cast<int64_t>(valid ? gr : 0) * row_stride + c * 8;
    cp_async16(sb + swz<D>(r, c * 8), src, valid);
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment (16x16, row-major source [rows][D]) at (r0, c0).
template <int D>
__device__ __forceinline__ void lda(uint32_t base, int r0, int c0, int lane, uint32_t (&a)[4]) {
  const int r = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int c = c0 + (lane >> 4) * 8;
  ldsm_x4(base + swz<D>(r, c), a[0], a[1], a[2], a[3]);
}
// A fragment from a transposed source: smem holds A^T as [k][m] rows.
template <int D>
__device__ __forceinline__ void lda_t(uint32_t base, int m0, int k0, int lane, uint32_t (&a)[4]) {
  const int r = k0 + (lane & 7) + (lane >> 4) * 8;
  const int c = m0 + ((lane >> 3) & 1) * 8;
  ldsm_x4_t(base + swz<D>(r, c), a[0], a[1], a[2], a[3]);
}
// Two B fragments (n-tiles n0, n0+8) from a source stored [n][k] (k contiguous).
template <int D>
__device__ __forceinline__ void ldb_nk(uint32_t base, int n0, int k0, int lane, uint32_t (&b)[4]) {
  const int r = n0 + (lane & 7) + (lane >> 4) * 8;
  const int c = k0 + ((lane >> 3) & 1) * 8;
  ldsm_x4(base + swz<D>(r, c), b[0], b[1], b[2], b[3]);
}
// Two B fragments (n-tiles n0, n0+8) from a source stored [k][n] (n contiguous).
template <int D>
__device__ __forceinline__ void ldb_kn(uint32_t base, int k0, int n0, int lane, uint32_t (&b)[4]) {
  const int r = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int c = n0 + (lane >> 4) * 8;
  ldsm_x4_t(base + swz<D>(r, c), b[0], b[1], b[2], b[3]);
}

struct AttnParams {
  const bf16* q;
  const bf16* k;
  const bf16* v;
  bf16* o;
  float* lse;
  const bf16* dout;  // backward only: dO [B,S,Hq,Dv] contiguous
  const float* delta;  // backward only: [B,Hq,S]
  float* dq_acc;       // backward only: [B,Hq,S,Dqk] fp32
  bf16* dq;            // backward only: [B,S,Hq,Dqk] strided
  bf16* dk;            // backward only: [B,S,Hkv,Dqk] strided
  bf16* dv;            // backward only: [B,S,Hkv,Dv] strided
  int64_t dq_sb, dq_ss, dq_sh;
  int64_t dk_sb, dk_ss, dk_sh;
  int64_t dv_sb, dv_ss, dv_sh;
  int64_t q_sb, q_ss, q_sh;
  int64_t k_sb, k_ss, k_sh;
  int64_t v_sb, v_ss, v_sh;
  int B, S, Hq, Hkv;
  float scale;
  float scale_log2;
  int causal;
};

// ================================================================ forward
template <int DQK, int DV>
struct FwdCfg {
  static constexpr int BM = 128, BN = 64, NT = 256;
  static constexpr int SMEM = (BM * DQK + 2 * BN * DQK + 2 * BN * DV) * 2;
};

template <int DQK, int DV>
__global__ void __launch_bounds__(256, 1) flash_fwd_kernel(AttnParams p) {
  using Cfg = FwdCfg<DQK, DV>;
  constexpr int BM = Cfg::BM, BN = Cfg::BN, NT = Cfg::NT;
  extern __shared__ __align__(128) uint8_t smem_attn[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_attn);
  bf16* sK = sQ + BM * DQK;
  bf16* sV = sK + 2 * BN * DQK;

  const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int q0 = qb * BM;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bf16* qg = p.q + b * p.q_sb + h * p.q_sh;
  const bf16* kg = p.k + b * p.k_sb + hk * p.k_sh;
  const bf16* vg = p.v + b * p.v_sb + hk * p.v_sh;

  const int nkb_all = (p.S + BN - 1) / BN;
  const int nkb = p.causal ? min(nkb_all, (q0 + BM - 1) / BN + 1) : nkb_all;

  load_tile<BM, DQK, NT>(sQ, qg, p.q_ss, q0, p.S, tid);
  load_tile<BN, DQK, NT>(sK, kg, p.k_ss, 0, p.S, tid);
  load_tile<BN, DV, NT>(sV, vg, p.v_ss, 0, p.S, tid);
  cp_async_commit();

  float o_acc[DV / 8][4];
#pragma unroll
  for (int i = 0; i < DV / 8; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  uint32_t qf[DQK / 16][4];

  const int r0 = warp * 16;
  const int row_a = q0 + r0 + (lane >> 2);
  const int row_b = row_a + 8;
  const uint32_t sQb = smem_u32(sQ);

  for (int kb = 0; kb < nkb; ++kb) {
    if (kb + 1 < nkb) {
      const int nb = (kb + 1) & 1;
      load_tile<BN, DQK, NT>(sK + nb * BN * DQK, kg, p.k_ss, (kb + 1) * BN, p.S, tid);
      load_tile<BN, DV, NT>(sV + nb * BN * DV, vg, p.v_ss, (kb + 1) * BN, p.S, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < DQK / 16; ++ks) lda<DQK>(sQb, r0, ks * 16, lane, qf[ks]);
    }
    const uint32_t sKb = smem_u32(sK + (kb & 1) * BN * DQK);
    const uint32_t sVb = smem_u32(sV + (kb & 1) * BN * DV);

    float s[BN / 8][4];
#pragma unroll
    for (int i = 0; i < BN / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DQK / 16; ++ks) {
#pragma unroll
      for (int n2 = 0; n2 < BN / 16; ++n2) {
        uint32_t bf[4];
        ldb_nk<DQK>(sKb, n2 * 16, ks * 16, lane, bf);
        mma16816(s[2 * n2], qf[ks], bf[0], bf[1]);
        mma16816(s[2 * n2 + 1], qf[ks], bf[2], bf[3]);
      }
    }
    // scale, mask, online softmax
    const int key0 = kb * BN + 2 * (lane & 3);
    const bool need_mask = (kb * BN + BN > p.S) || (p.causal && kb * BN + BN - 1 > q0 + r0);
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < BN / 8; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int key = key0 + nt * 8 + j;
        float va = s[nt][j] * p.scale_log2, vb = s[nt][2 + j] * p.scale_log2;
        if (need_mask) {
          if (key >= p.S || (p.causal && key > row_a)) va = -INFINITY;
          if (key >= p.S || (p.causal && key > row_b)) vb = -INFINITY;
        }
        s[nt][j] = va;
        s[nt][2 + j] = vb;
        mx_a = fmaxf(mx_a, va);
        mx_b = fmaxf(mx_b, vb);
      }
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float base_a = (mn_a == -INFINITY) ? 0.f : mn_a;
    const float base_b = (mn_b == -INFINITY) ? 0.f : mn_b;
    const float alpha_a = exp2f(m_a - base_a), alpha_b = exp2f(m_b - base_b);
    m_a = mn_a;
    m_b = mn_b;
    float sum_a = 0.f, sum_b = 0.f;
    uint32_t pa[BN / 16][4];
#pragma unroll
    for (int nt = 0; nt < BN / 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - base_a), p1 = exp2f(s[nt][1] - base_a);
      const float p2 = exp2f(s[nt][2] - base_b), p3 = exp2f(s[nt][3] - base_b);
      sum_a += p0 + p1;
      sum_b += p2 + p3;
      const int j = nt >> 1;
      if ((nt & 1) == 0) {
        pa[j][0] = pack_bf16x2(p0, p1);
        pa[j][1] = pack_bf16x2(p2, p3);
      } else {
        pa[j][2] = pack_bf16x2(p0, p1);
        pa[j][3] = pack_bf16x2(p2, p3);
      }
    }
    l_a = l_a * alpha_a + sum_a;
    l_b = l_b * alpha_b + sum_b;
#pragma unroll
    for (int i = 0; i < DV / 8; ++i) {
      o_acc[i][0] *= alpha_a;
      o_acc[i][1] *= alpha_a;
      o_acc[i][2] *= alpha_b;
      o_acc[i][3] *= alpha_b;
    }
#pragma unroll
    for (int j = 0; j < BN / 16; ++j) {
#pragma unroll
      for (int d2 = 0; d2 < DV / 16; ++d2) {
        uint32_t bf[4];
        ldb_kn<DV>(sVb, j * 16, d2 * 16, lane, bf);
        mma16816(o_acc[2 * d2], pa[j], bf[0], bf[1]);
        mma16816(o_acc[2 * d2 + 1], pa[j], bf[2], bf[3]);
      }
    }
    __syncthreads();
  }

  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f;
  const float inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  const int64_t o_ss = static_cast<int64_t>(p.Hq) * DV;
  bf16* og = p.o + static_cast<int64_t>(b) * p.S * o_ss + static_cast<int64_t>(h) * DV;
  const int c0 = 2 * (lane & 3);
  if (row_a < p.S) {
#pragma unroll
    for (int i = 0; i < DV / 8; ++i)
      *reinterpret_cast<uint32_t*>(og + row_a * o_ss + i * 8 + c0) = pack_bf16x2(o_acc[i][0] * inv_a, o_acc[i][1] * inv_a);
  }
  if (row_b < p.S) {
#pragma unroll
    for (int i = 0; i < DV / 8; ++i)
      *reinterpret_cast<uint32_t*>(og + row_b * o_ss + i * 8 + c0) = pack_bf16x2(o_acc[i][2] * inv_b, o_acc[i][3] * inv_b);
  }
  if ((lane & 3) == 0) {
    float* lg = p.lse + (static_cast<int64_t>(b) * p.Hq + h) * p.S;
    if (row_a < p.S) lg[row_a] = m_a + log2f(l_a);
    if (row_b < p.S) lg[row_b] = m_b + log2f(l_b);
  }
}

// ================================================================ backward
// delta[b,h,s] = sum_d dO * O
__global__ void attn_bwd_delta_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ out,
                                      float* __restrict__ delta, int B, int S, int H, int D) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= static_cast<int64_t>(B) * S * H) return;
  const bf16* a = dout + row * D;
  const bf16* c = out + row * D;
  float acc = 0.f;
  for (int i = lane * 2; i < D; i += 64) {
    const __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162*>(a + i);
    const __nv_bfloat162 y = *reinterpret_cast<const __nv_bfloat162*>(c + i);
    acc += __bfloat162float(x.x) * __bfloat162float(y.x) + __bfloat162float(x.y) * __bfloat162float(y.y);
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const int h = row % H;
    const int64_t bs = row / H;
    const int s = bs % S;
    const int bb = bs / S;
    delta[(static_cast<int64_t>(bb) * H + h) * S + s] = acc;
  }
}

// dq[b,s,h,:] = bf16(acc[b,h,s,:] * scale) (dq strided)
// delta with 16-byte loads: half a warp per (b, s, h) row, 8 elements per lane per step; rows are
// grid-strided so each warp keeps two rows' loads in flight. Needs D % 8 == 0 and 16-byte aligned rows.
__global__ void __launch_bounds__(256) attn_bwd_delta_vec_kernel(const bf16* __restrict__ dout,
                                                                 const bf16* __restrict__ out,
                                                                 float* __restrict__ delta, int B, int S, int H,
                                                                 int D) {
  const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
  const int64_t rows = static_cast<int64_t>(B) * S * H;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); 2 * w < rows;
       w += nwarps) {
    const int64_t row = 2 * w + half;
    const bool live = row < rows;
    float acc = 0.f;
    if (live) {
      const bf16* a = dout + row * D;
      const bf16* c = out + row * D;
      for (int i = hl * 8; i < D; i += 128) {
        const uint4 x = *reinterpret_cast<const uint4*>(a + i);
        const uint4 y = *reinterpret_cast<const uint4*>(c + i);
        acc += bf16_lo(x.x) * bf16_lo(y.x) + bf16_hi(x.x) * bf16_hi(y.x) + bf16_lo(x.y) * bf16_lo(y.y) +
               bf16_hi(x.y) * bf16_hi(y.y) + bf16_lo(x.z) * bf16_lo(y.z) + bf16_hi(x.z) * bf16_hi(y.z) +
               bf16_lo(x.w) * bf16_lo(y.w) + bf16_hi(x.w) * bf16_hi(y.w);
      }
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (live && hl == 0) {
      const int h = static_cast<int>(row % H);
      const int64_t bs = row / H;
      const int s = static_cast<int>(bs % S);
      const int64_t bb = bs / S;
      delta[(bb * H + h) * S + s] = acc;
    }
  }
}

__global__ void attn_bwd_dq_convert_kernel(const float* __restrict__ acc, bf16* __restrict__ dq, int B, int S, int H,
                                           int D, float scale, int64_t sb, int64_t ss, int64_t sh) {
  const int64_t total = static_cast<int64_t>(B) * S * H * D;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int d = i % D;
    const int64_t r = i / D;
    const int h = r % H;
    const int64_t bs = r / H;
    const int s = bs % S;
    const int bb = bs / S;
    dq[bb * sb + s * ss + h * sh + d] = __float2bfloat16(acc[((static_cast<int64_t>(bb) * H + h) * S + s) * D + d] * scale);
  }
}

// The same conversion, 8 head-dim elements per thread: two 16-byte loads of the fp32 accumulator,
// one 16-byte bf16 store, threads ordered like the output rows (b, s, h) so the stores coalesce.
// Needs D % 8 == 0 and 16-byte aligned output rows.
__global__ void __launch_bounds__(256) attn_bwd_dq_convert_vec_kernel(const float* __restrict__ acc,
                                                                      bf16* __restrict__ dq, int B, int S, int H,
                                                                      int D, float scale, int64_t sb, int64_t ss,
                                                                      int64_t sh) {
  const int cpr = D / 8;  // chunks per (b, s, h) row
  const int64_t total = static_cast<int64_t>(B) * S * H * cpr;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % cpr);
    const int64_t r = i / cpr;
    const int h = static_cast<int>(r % H);
    const int64_t bs = r / H;
    const int s = static_cast<int>(bs % S);
    const int64_t bb = bs / S;
    const float4* src = reinterpret_cast<const float4*>(acc + ((bb * H + h) * S + s) * D + c * 8);
    const float4 a = src[0], b = src[1];
    uint4 o;
    o.x = pack_bf16x2(a.x * scale, a.y * scale);
    o.y = pack_bf16x2(a.z * scale, a.w * scale);
    o.z = pack_bf16x2(b.x * scale, b.y * scale);
    o.w = pack_bf16x2(b.z * scale, b.w * scale);
    *reinterpret_cast<uint4*>(dq + bb * sb + s * ss + h * sh + c * 8) = o;
  }
}

template <int DQK, int DV>
struct BwdCfg {
  static constexpr int BN = 128;                  // keys per CTA (8 warps x 16)
  static constexpr int BM = DQK > 128 ? 32 : 64;  // queries per iteration
  static constexpr int NT = 256;
  static constexpr int SK = BN * DQK * 2, SV = BN * DV * 2;
  static constexpr int SQ = BM * DQK * 2, SDO = BM * DV * 2;
  static constexpr int SDS = BN * BM * 2;
  static constexpr int SSTAGE = BM * DQK * 4;
  static constexpr int SMEM = SK + SV + 2 * SQ + 2 * SDO + SDS + SSTAGE + 2 * 2 * BM * 4;
};

template <int DQK, int DV>
__global__ void __launch_bounds__(256, 1) flash_bwd_kernel(AttnParams p) {
  using Cfg = BwdCfg<DQK, DV>;
  constexpr int BN = Cfg::BN, BM = Cfg::BM, NT = Cfg::NT;
  extern __shared__ __align__(128) uint8_t smem_attn[];
  uint8_t* sp = smem_attn;
  bf16* sK = reinterpret_cast<bf16*>(sp);
  sp += Cfg::SK;
  bf16* sV = reinterpret_cast<bf16*>(sp);
  sp += Cfg::SV;
  bf16* sQ = reinterpret_cast<bf16*>(sp);
  sp += 2 * Cfg::SQ;
  bf16* sdO = reinterpret_cast<bf16*>(sp);
  sp += 2 * Cfg::SDO;
  bf16* sdS = reinterpret_cast<bf16*>(sp);
  sp += Cfg::SDS;
  float* sStage = reinterpret_cast<float*>(sp);
  sp += Cfg::SSTAGE;
  float* sLse = reinterpret_cast<float*>(sp);  // [2][BM]
  float* sDel = sLse + 2 * BM;                 // [2][BM]

  const int kb = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = p.Hq / p.Hkv;
  const int key0 = kb * BN;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bf16* kg = p.k + b * p.k_sb + hk * p.k_sh;
  const bf16* vg = p.v + b * p.v_sb + hk * p.v_sh;
  const int64_t do_ss = static_cast<int64_t>(p.Hq) * DV;

  load_tile<BN, DQK, NT>(sK, kg, p.k_ss, key0, p.S, tid);
  load_tile<BN, DV, NT>(sV, vg, p.v_ss, key0, p.S, tid);

  const int nqb = (p.S + BM - 1) / BM;
  const int qb0 = p.causal ? key0 / BM : 0;
  const int per_head = nqb - qb0;
  const int n_it = per_head * G;

  auto issue = [&](int it, int buf) {
    const int h = hk * G + it / per_head;
    const int qb = qb0 + it % per_head;
    const int q0 = qb * BM;
    const bf16* qg = p.q + b * p.q_sb + h * p.q_sh;
    const bf16* dg = p.dout + static_cast<int64_t>(b) * p.S * do_ss + static_cast<int64_t>(h) * DV;
    load_tile<BM, DQK, NT>(sQ + buf * BM * DQK, qg, p.q_ss, q0, p.S, tid);
    load_tile<BM, DV, NT>(sdO + buf * BM * DV, dg, do_ss, q0, p.S, tid);
    if (tid < BM) {
      const int q = q0 + tid;
      const int64_t base = (static_cast<int64_t>(b) * p.Hq + h) * p.S;
      sLse[buf * BM + tid] = q < p.S ? p.lse[base + q] : INFINITY;
      sDel[buf * BM + tid] = q < p.S ? p.delta[base + q] : 0.f;
    }
  };

  if (n_it > 0) issue(0, 0);
  cp_async_commit();

  float dk_acc[DQK / 8][4], dv_acc[DV / 8][4];
#pragma unroll
  for (int i = 0; i < DQK / 8; ++i) dk_acc[i][0] = dk_acc[i][1] = dk_acc[i][2] = dk_acc[i][3] = 0.f;
#pragma unroll
  for (int i = 0; i < DV / 8; ++i) dv_acc[i][0] = dv_acc[i][1] = dv_acc[i][2] = dv_acc[i][3] = 0.f;

  const int kr0 = warp * 16;                          // this warp's keys within the block
  const int key_a = key0 + kr0 + (lane >> 2), key_b = key_a + 8;
  const uint32_t sKb = smem_u32(sK), sVb = smem_u32(sV), sdSb = smem_u32(sdS);
  // dQ tile split: (BM/16) row groups x (8 / (BM/16)) column slices.
  constexpr int RG = BM / 16;
  constexpr int CS = 8 / RG;
  constexpr int DQC = DQK / CS;  // columns per warp
  const int dq_r0 = (warp % RG) * 16, dq_c0 = (warp / RG) * DQC;

  for (int it = 0; it < n_it; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_it) {
      issue(it + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int h = hk * G + it / per_head;
    const int q0 = (qb0 + it % per_head) * BM;
    const uint32_t sQb = smem_u32(sQ + buf * BM * DQK);
    const uint32_t sdOb = smem_u32(sdO + buf * BM * DV);
    const float* lse = sLse + buf * BM;
    const float* del = sDel + buf * BM;

    // S^T = K Q^T  (16 keys x BM queries per warp)
    float st[BM / 8][4];
#pragma unroll
    for (int i = 0; i < BM / 8; ++i) st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DQK / 16; ++ks) {
      uint32_t af[4];
      lda<DQK>(sKb, kr0, ks * 16, lane, af);
#pragma unroll
      for (int n2 = 0; n2 < BM / 16; ++n2) {
        uint32_t bf[4];
        ldb_nk<DQK>(sQb, n2 * 16, ks * 16, lane, bf);
        mma16816(st[2 * n2], af, bf[0], bf[1]);
        mma16816(st[2 * n2 + 1], af, bf[2], bf[3]);
      }
    }
    // P^T = exp2(S^T * scale_log2 - lse[q]), masked
    const bool need_mask = (q0 + BM > p.S) || (key0 + BN > p.S) || (p.causal && q0 < key0 + kr0 + 16);
#pragma unroll
    for (int nt = 0; nt < BM / 8; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int ql = nt * 8 + 2 * (lane & 3) + j;
        const int q = q0 + ql;
        float pa = exp2f(st[nt][j] * p.scale_log2 - lse[ql]);
        float pb = exp2f(st[nt][2 + j] * p.scale_log2 - lse[ql]);
        if (need_mask) {
          if (q >= p.S || key_a >= p.S || (p.causal && q < key_a)) pa = 0.f;
          if (q >= p.S || key_b >= p.S || (p.causal && q < key_b)) pb = 0.f;
        }
        st[nt][j] = pa;
        st[nt][2 + j] = pb;
      }
    }
    // dV += P^T dO
    uint32_t pf[BM / 16][4];
#pragma unroll
    for (int j = 0; j < BM / 16; ++j) {
      pf[j][0] = pack_bf16x2(st[2 * j][0], st[2 * j][1]);
      pf[j][1] = pack_bf16x2(st[2 * j][2], st[2 * j][3]);
      pf[j][2] = pack_bf16x2(st[2 * j + 1][0], st[2 * j + 1][1]);
      pf[j][3] = pack_bf16x2(st[2 * j + 1][2], st[2 * j + 1][3]);
    }
#pragma unroll
    for (int j = 0; j < BM / 16; ++j) {
#pragma unroll
      for (int d2 = 0; d2 < DV / 16; ++d2) {
        uint32_t bf[4];
        ldb_kn<DV>(sdOb, j * 16, d2 * 16, lane, bf);
        mma16816(dv_acc[2 * d2], pf[j], bf[0], bf[1]);
        mma16816(dv_acc[2 * d2 + 1], pf[j], bf[2], bf[3]);
      }
    }
    // dP^T = V dO^T
    float dpt[BM / 8][4];
#pragma unroll
    for (int i = 0; i < BM / 8; ++i) dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DV / 16; ++ks) {
      uint32_t af[4];
      lda<DV>(sVb, kr0, ks * 16, lane, af);
#pragma unroll
      for (int n2 = 0; n2 < BM / 16; ++n2) {
        uint32_t bf[4];
        ldb_nk<DV>(sdOb, n2 * 16, ks * 16, lane, bf);
        mma16816(dpt[2 * n2], af, bf[0], bf[1]);
        mma16816(dpt[2 * n2 + 1], af, bf[2], bf[3]);
      }
    }
    // dS^T = P^T * (dP^T - delta[q])
    uint32_t dsf[BM / 16][4];
#pragma unroll
    for (int nt = 0; nt < BM / 8; ++nt) {
      const int ql = nt * 8 + 2 * (lane & 3);
      const float d0 = st[nt][0] * (dpt[nt][0] - del[ql]);
      const float d1 = st[nt][1] * (dpt[nt][1] - del[ql + 1]);
      const float d2v = st[nt][2] * (dpt[nt][2] - del[ql]);
      const float d3 = st[nt][3] * (dpt[nt][3] - del[ql + 1]);
      const int j = nt >> 1;
      if ((nt & 1) == 0) {
        dsf[j][0] = pack_bf16x2(d0, d1);
        dsf[j][1] = pack_bf16x2(d2v, d3);
      } else {
        dsf[j][2] = pack_bf16x2(d0, d1);
        dsf[j][3] = pack_bf16x2(d2v, d3);
      }
      // dS^T to shared memory [keys][queries] for the dQ product.
      const int kr = kr0 + (lane >> 2);
      *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(sdS) + swz<BM>(kr, ql)) = pack_bf16x2(d0, d1);
      *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(sdS) + swz<BM>(kr + 8, ql)) = pack_bf16x2(d2v, d3);
    }
    // dK += dS^T Q
#pragma unroll
    for (int j = 0; j < BM / 16; ++j) {
#pragma unroll
      for (int d2 = 0; d2 < DQK / 16; ++d2) {
        uint32_t bf[4];
        ldb_kn<DQK>(sQb, j * 16, d2 * 16, lane, bf);
        mma16816(dk_acc[2 * d2], dsf[j], bf[0], bf[1]);
        mma16816(dk_acc[2 * d2 + 1], dsf[j], bf[2], bf[3]);
      }
    }
    // The previous bulk reduction must have finished reading the staging tile.
    if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    __syncthreads();
    // dQ partial = dS K : warp computes rows [dq_r0, +16) x cols [dq_c0, +DQC)
    {
      float acc[DQC / 8][4];
#pragma unroll
      for (int i = 0; i < DQC / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < BN / 16; ++ks) {
        uint32_t af[4];
        lda_t<BM>(sdSb, dq_r0, ks * 16, lane, af);
#pragma unroll
        for (int d2 = 0; d2 < DQC / 16; ++d2) {
          uint32_t bf[4];
          ldb_kn<DQK>(sKb, ks * 16, dq_c0 + d2 * 16, lane, bf);
          mma16816(acc[2 * d2], af, bf[0], bf[1]);
          mma16816(acc[2 * d2 + 1], af, bf[2], bf[3]);
        }
      }
      const int ra = dq_r0 + (lane >> 2);
#pragma unroll
      for (int i = 0; i < DQC / 8; ++i) {
        const int c = dq_c0 + i * 8 + 2 * (lane & 3);
        *reinterpret_cast<float2*>(sStage + ra * DQK + c) = make_float2(acc[i][0], acc[i][1]);
        *reinterpret_cast<float2*>(sStage + (ra + 8) * DQK + c) = make_float2(acc[i][2], acc[i][3]);
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      const int valid = min(BM, p.S - q0);
      float* dst = p.dq_acc + ((static_cast<int64_t>(b) * p.Hq + h) * p.S + q0) * DQK;
      const uint32_t bytes = static_cast<uint32_t>(valid * DQK * 4);
      asm volatile(
          "cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(dst),
          "r"(smem_u32(sStage)), "r"(bytes)
          : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
  if (tid == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");

  // write dK (scaled) and dV
  const int64_t dk_ss = p.dk_ss, dv_ss = p.dv_ss;
  bf16* dkg = p.dk + b * p.dk_sb + hk * p.dk_sh;
  bf16* dvg = p.dv + b * p.dv_sb + hk * p.dv_sh;
  const int c0 = 2 * (lane & 3);
  if (key_a < p.S) {
#pragma unroll
    for (int i = 0; i < DQK / 8; ++i)
      *reinterpret_cast<uint32_t*>(dkg + key_a * dk_ss + i * 8 + c0) =
          pack_bf16x2(dk_acc[i][0] * p.scale, dk_acc[i][1] * p.scale);
#pragma unroll
    for (int i = 0; i < DV / 8; ++i)
      *reinterpret_cast<uint32_t*>(dvg + key_a * dv_ss + i * 8 + c0) = pack_bf16x2(dv_acc[i][0], dv_acc[i][1]);
  }
  if (key_b < p.S) {
#pragma unroll
    for (int i = 0; i < DQK / 8; ++i)
      *reinterpret_cast<uint32_t*>(dkg + key_b * dk_ss + i * 8 + c0) =
          pack_bf16x2(dk_acc[i][2] * p.scale, dk_acc[i][3] * p.scale);
#pragma unroll
    for (int i = 0; i < DV / 8; ++i)
      *reinterpret_cast<uint32_t*>(dvg + key_b * dv_ss + i * 8 + c0) = pack_bf16x2(dv_acc[i][2], dv_acc[i][3]);
  }
}

// ================================================================ host
static AttnParams make_params(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                              bool causal) {
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "flash_attn: 4-D [B,S,H,D] tensors");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "flash_attn: bf16");
  TORCH_CHECK(q.stride(3) == 1 && k.stride(3) == 1 && v.stride(3) == 1, "flash_attn: head dim must be contiguous");
  TORCH_CHECK(k.size(1) == q.size(1) && v.size(1) == q.size(1), "flash_attn: self-attention only (Sq == Sk)");
  TORCH_CHECK(q.size(2) % k.size(2) == 0 && k.size(2) == v.size(2), "flash_attn: GQA head ratio");
  for (const auto* t : {&q, &k, &v}) {
    TORCH_CHECK((reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0, "flash_attn: 16B aligned base");
    TORCH_CHECK(t->stride(0) % 8 == 0 && t->stride(1) % 8 == 0 && t->stride(2) % 8 == 0, "flash_attn: 16B strides");
  }
  AttnParams p{};
  p.q = reinterpret_cast<const bf16*>(q.data_ptr());
  p.k = reinterpret_cast<const bf16*>(k.data_ptr());
  p.v = reinterpret_cast<const bf16*>(v.data_ptr());
  p.q_sb = q.stride(0); p.q_ss = q.stride(1); p.q_sh = q.stride(2);
  p.k_sb = k.stride(0); p.k_ss = k.stride(1); p.k_sh = k.stride(2);
  p.v_sb = v.stride(0); p.v_ss = v.stride(1); p.v_sh = v.stride(2);
  p.B = static_cast<int>(q.size(0));
  p.S = static_cast<int>(q.size(1));
  p.Hq = static_cast<int>(q.size(2));
  p.Hkv = static_cast<int>(k.size(2));
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  return p;
}

template <typename K>
static void set_smem(K kern, int bytes) {
  NTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

std::vector<at::Tensor> flash_attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                                       bool causal) {
  AttnParams p = make_params(q, k, v, scale, causal);
  const int DQK = static_cast<int>(q.size(3)), DV = static_cast<int>(v.size(3));
  auto o = at::empty({q.size(0), q.size(1), q.size(2), v.size(3)}, q.options());
  auto lse = at::empty({q.size(0), q.size(2), q.size(1)}, q.options().dtype(at::kFloat));
  p.o = reinterpret_cast<bf16*>(o.data_ptr());
  p.lse = lse.data_ptr<float>();
  if (p.S == 0 || p.B == 0) return {o, lse};
  auto stream = at::cuda::getCurrentCUDAStream();
#define NTB_FWD(DQ, DVV)                                                             \
  if (DQK == DQ && DV == DVV) {                                                      \
    using Cfg = FwdCfg<DQ, DVV>;                                                     \
    set_smem(flash_fwd_kernel<DQ, DVV>, Cfg::SMEM);                                  \
    dim3 grid((p.S + Cfg::BM - 1) / Cfg::BM, p.Hq, p.B);                             \
    flash_fwd_kernel<DQ, DVV><<<grid, Cfg::NT, Cfg::SMEM, stream>>>(p);              \
    NTB_LAUNCH_CHECK(1);                                                             \
    return {o, lse};                                                                 \
  }
  NTB_FWD(64, 64)
  NTB_FWD(128, 128)
  NTB_FWD(192, 128)
#undef NTB_FWD
  TORCH_CHECK(false, "flash_attn_fwd: unsupported head dims ", DQK, "/", DV);
}

// dq/dk/dv may be given as (strided) views to write into, e.g. the column
// slices of one fused dQKV buffer; otherwise they are allocated.
std::vector<at::Tensor> flash_attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                       const at::Tensor& v, const at::Tensor& out, const at::Tensor& lse, double scale,
                                       bool causal, const c10::optional<at::Tensor>& dq_opt,
                                       const c10::optional<at::Tensor>& dk_opt, const c10::optional<at::Tensor>& dv_opt) {
  AttnParams p = make_params(q, k, v, scale, causal);
  const int DQK = static_cast<int>(q.size(3)), DV = static_cast<int>(v.size(3));
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous(), "flash_attn_bwd: contiguous dO and O");
  auto dq = dq_opt.has_value() ? *dq_opt : at::empty({q.size(0), q.size(1), q.size(2), q.size(3)}, q.options());
  auto dk = dk_opt.has_value() ? *dk_opt : at::empty({k.size(0), k.size(1), k.size(2), k.size(3)}, k.options());
  auto dv = dv_opt.has_value() ? *dv_opt : at::empty({v.size(0), v.size(1), v.size(2), v.size(3)}, v.options());
  TORCH_CHECK(dq.sizes() == q.sizes() && dk.sizes() == k.sizes() && dv.sizes() == v.sizes(), "flash_attn_bwd: grad shapes");
  TORCH_CHECK(dq.stride(3) == 1 && dk.stride(3) == 1 && dv.stride(3) == 1, "flash_attn_bwd: grad head dim contiguous");
  if (p.S == 0 || p.B == 0) return {dq.zero_(), dk.zero_(), dv.zero_()};
  p.dq = reinterpret_cast<bf16*>(dq.data_ptr());
  p.dq_sb = dq.stride(0); p.dq_ss = dq.stride(1); p.dq_sh = dq.stride(2);
  p.dk_sb = dk.stride(0); p.dk_ss = dk.stride(1); p.dk_sh = dk.stride(2);
  p.dv_sb = dv.stride(0); p.dv_ss = dv.stride(1); p.dv_sh = dv.stride(2);
  auto delta = at::empty({q.size(0), q.size(2), q.size(1)}, q.options().dtype(at::kFloat));
  auto dq_acc = at::zeros({q.size(0), q.size(2), q.size(1), q.size(3)}, q.options().dtype(at::kFloat));
  auto stream = at::cuda::getCurrentCUDAStream();
  {
    const int64_t rows = static_cast<int64_t>(p.B) * p.S * p.Hq;
    const bool vec = DV % 8 == 0 && out.is_contiguous() && dout.is_contiguous() &&
                     (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(dout.data_ptr()) & 15) == 0;
    if (vec)
      attn_bwd_delta_vec_kernel<<<static_cast<int>(std::min<int64_t>((rows + 15) / 16, 148 * 8)), 256, 0, stream>>>(
          reinterpret_cast<const bf16*>(dout.data_ptr()), reinterpret_cast<const bf16*>(out.data_ptr()),
          delta.data_ptr<float>(), p.B, p.S, p.Hq, DV);
    else
      attn_bwd_delta_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(reinterpret_cast<const bf16*>(dout.data_ptr()),
                                                                 reinterpret_cast<const bf16*>(out.data_ptr()),
                                                                 delta.data_ptr<float>(), p.B, p.S, p.Hq, DV);
  }
  p.dout = reinterpret_cast<const bf16*>(dout.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dk = reinterpret_cast<bf16*>(dk.data_ptr());
  p.dv = reinterpret_cast<bf16*>(dv.data_ptr());
  bool launched = false;
  if (flash_attn_bwd_tc_supported(DQK, DV) && std::getenv("NTB_ATTN_BWD_LEGACY") == nullptr) {
    flash_attn_bwd_tc_launch(q, k, v, dout, lse, delta, dq_acc, dk, dv, scale, causal);
    launched = true;
  }
#define NTB_BWD(DQ, DVV)                                                             \
  if (!launched && DQK == DQ && DV == DVV) {                                         \
    using Cfg = BwdCfg<DQ, DVV>;                                                     \
    set_smem(flash_bwd_kernel<DQ, DVV>, Cfg::SMEM);                                  \
    dim3 grid((p.S + Cfg::BN - 1) / Cfg::BN, p.Hkv, p.B);                            \
    flash_bwd_kernel<DQ, DVV><<<grid, Cfg::NT, Cfg::SMEM, stream>>>(p);              \
    NTB_LAUNCH_CHECK(2);                                                             \
    launched = true;                                                                 \
  }
  NTB_BWD(64, 64)
  NTB_BWD(128, 128)
  NTB_BWD(192, 128)
#undef NTB_BWD
  TORCH_CHECK(launched, "flash_attn_bwd: unsupported head dims ", DQK, "/", DV);
  const int64_t total = static_cast<int64_t>(p.B) * p.S * p.Hq * DQK;
  const bool vec = DQK % 8 == 0 && p.dq_sb % 8 == 0 && p.dq_ss % 8 == 0 && p.dq_sh % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(p.dq) & 15) == 0;
  if (vec) {
    const int blocks = static_cast<int>(std::min<int64_t>((total / 8 + 255) / 256, 148 * 16));
    attn_bwd_dq_convert_vec_kernel<<<blocks, 256, 0, stream>>>(dq_acc.data_ptr<float>(), p.dq, p.B, p.S, p.Hq, DQK,
                                                               p.scale, p.dq_sb, p.dq_ss, p.dq_sh);
  } else {
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
    attn_bwd_dq_convert_kernel<<<blocks, 256, 0, stream>>>(dq_acc.data_ptr<float>(), p.dq, p.B, p.S, p.Hq, DQK,
                                                           p.scale, p.dq_sb, p.dq_ss, p.dq_sh);
  }
  NTB_LAUNCH_CHECK(1);
  return {dq, dk, dv};
}

}  // namespace ntb
