// Persistent warp-specialised bf16 GEMM for sm_100a on the 5th-gen tensor cores.
//
//   C[M,N] = alpha * op(A)[M,K] . op(B)[N,K]^T  (+ bias[N]) (+ C)
//
// op(A) is either A stored [M,K] (K-major) or A stored [K,M] (M-major); op(B)
// is B stored [N,K] (K-major) or [K,N] (N-major). The three linear-layer
// GEMMs map onto it without any transpose copy:
//   forward  Y  = X . W^T   : A=X  [T,in]  K-major, B=W [out,in] K-major
//   dgrad    dX = dY . W    : A=dY [T,out] K-major, B=W [out,in] N-major
//   wgrad    dW = dY^T . X  : A=dY [T,out] M-major, B=X [T,in]  N-major
//
// Design (one CTA per SM, 192 threads):
//   warp 0      TMA producer: 128B-swizzled tiles into a STAGES-deep SMEM ring
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma 128xBNx16
//               into a TMEM accumulator; owns the TMEM allocation
//   warps 2..5  epilogue: tcgen05.ld TMEM -> registers -> fused bias /
//               accumulate / cast -> global
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the main loop of tile i+1. Tiles are walked in
// M-grouped order so one wave of CTAs shares A and B panels in the 126 MB L2.
// Every wait is bounded (see common.cuh) and reports into a status word.
//
// Reference parity: replaces the F.linear / autograd matmuls of
// src/layers.py:628-632, 1358-1360, 1484 (eager cuBLAS in the reference).
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "host_utils.h"
#include "peer.cuh"

namespace ntb {

struct GemmParams {
  int M, N, K;
  void* C;
  long ldc;
  const __nv_bfloat16* bias;
  float alpha;
  int accumulate;  // 1: C = result + C (C read in its own dtype)
  int c_f32;       // 1: C is fp32, else bf16
  int* status;
  // Grouped (mixture-of-experts) modes, see gemm_grouped_bf16:
  const int* offsets;  // [groups + 1] row offsets, multiples of 128
  int groups;
  int b_group_rows;    // rows of one group's slice of the stacked B (mode 1)
  long m_limit;        // rows of C that exist (mode 2: per-group output rows)
  long c_group_stride; // mode 2: rows of C between consecutive groups' blocks (0 = M, a dense stack)
  // Plain GEMM with an fp32 accumulated C only: K is cut into `splits` slices (1 = no split). Each
  // (tile, slice) unit adds its partial product into C with vector atomics, so the sum's
  // rounding order varies from run to run (fp32 low bits only).
  int splits;
  // Publication (plain GEMM, optional): when pub_n > 0, the last CTA to finish makes the whole C
  // visible system-wide (fence.sc.sys) and stores pub_epoch into pub_flag[0..pub_n) - the epoch
  // words of the peers that read C over NVLink. pub_ctr: a device u32 that is zero at rest.
  unsigned long long* pub_flag[8];
  int pub_n;
  unsigned long long pub_epoch;
  unsigned int* pub_ctr;
};

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int STAGE_BYTES = 4 * 8192;  // epilogue staging: 32 rows x 64 fp32 per epilogue warp
  static constexpr int SMEM_BYTES =
      1024 /*align slack*/ + STAGES * (A_BYTES + B_BYTES) + STAGE_BYTES + 256 /*barriers*/;
};

// Grouped GEMM modes (template parameter GM):
//   0  plain GEMM
//   1  M-grouped (expert forward / input gradient): rows of A and C are grouped by
//      expert, each group padded to a multiple of 128 rows; B is a stack of per-expert
//      matrices and a tile reads the slice of the expert that owns its first row.
//   2  K-grouped (expert weight gradient): the output is a stack of per-expert
//      [M, N] blocks; tile = (expert, m, n) and K runs over that expert's rows.
struct TileInfo {
  int mb, nb, group, kb0, nkb, slice;
};

__device__ __forceinline__ int group_of_row(const int* offsets, int groups, int row) {
  int lo = 0, hi = groups - 1;  // last g with offsets[g] <= row
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(offsets + mid) <= row) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  constexpr int GROUP = 16;
  const int per_group = GROUP * num_n;
  const int g = tile / per_group;
  const int first_m = g * GROUP;
  const int gm = min(GROUP, num_m - first_m);
  const int r = tile - g * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

// Epilogue of one warp's 32 accumulator rows (TMEM lanes) of a 128 x BN tile.
// Each 64-column group is read from TMEM (the lane's row), scaled and biased in
// fp32, staged through the warp's 8 KB of shared memory (16-byte chunks
// XOR-swizzled by row) and written row-contiguously: a warp instruction stores
// 4 rows x 128 B (bf16) or 2 rows x 256 B (fp32) instead of 32 scattered
// 16-byte pieces. `accumulate` adds the previous C in fp32 before the single
// final rounding. m0: first row of the warp; n0: first column of the tile.
template <int BN>
__device__ __forceinline__ void epilogue_tile(uint32_t t_row, float* stage, const GemmParams& p, long m0, int n0,
                                              bool vec_ok, long m_end, bool red = false) {
  const int lane = threadIdx.x & 31;
  const bool f32 = p.c_f32 != 0;
  // red: a K-slice of a split GEMM (fp32 C) - the partial is added with atomics, C is not read.
  const bool acc = p.accumulate != 0 && !red;
#pragma unroll 1
  for (int g = 0; g < BN; g += 64) {
    const int cg = n0 + g;
    if (cg >= p.N) break;  // warp-uniform
    // With accumulation, the previous C of this 64-column group is requested first so
    // its DRAM latency overlaps the TMEM read and the staging below.
    float4 old[16];
    if (acc) {
      if (f32) {
#pragma unroll
        for (int it = 0; it < 16; ++it) {
          const int row = it * 2 + (lane >> 4), col = cg + (lane & 15) * 4;
          const long m = m0 + row;
          old[it] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (m < m_end && vec_ok && col + 4 <= p.N && (p.ldc & 3) == 0)
            old[it] = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.C) + m * p.ldc + col);
        }
      } else {
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int row = it * 4 + (lane >> 3), col = cg + (lane & 7) * 8;
          const long m = m0 + row;
          old[it] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (m < m_end && vec_ok && col + 8 <= p.N)
            old[it] = *reinterpret_cast<const float4*>(reinterpret_cast<const __nv_bfloat16*>(p.C) + m * p.ldc + col);
        }
      }
    }
    uint32_t r0[32], r1[32];
    tmem_ld32(t_row + g, r0);
    tmem_ld32(t_row + g + 32, r1);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float4 v;
      float* w = &v.x;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = j * 4 + u;
        const uint32_t bits = c < 32 ? r0[c] : r1[c - 32];
        float x = __uint_as_float(bits) * p.alpha;
        if (p.bias != nullptr && !red && cg + c < p.N) x += __bfloat162float(p.bias[cg + c]);
        w[u] = x;
      }
      *reinterpret_cast<float4*>(stage + lane * 64 + ((j ^ (lane & 15)) * 4)) = v;
    }
    __syncwarp();
    if (f32) {
      float* C = reinterpret_cast<float*>(p.C);
#pragma unroll
      for (int it = 0; it < 16; ++it) {
        const int row = it * 2 + (lane >> 4), ch = lane & 15;
        const long m = m0 + row;
        const int col = cg + ch * 4;
        if (m >= m_end || col >= p.N) continue;
        float4 v = *reinterpret_cast<const float4*>(stage + row * 64 + ((ch ^ (row & 15)) * 4));
        float* dst = C + m * p.ldc + col;
        if (red) {
          if (vec_ok && col + 4 <= p.N && (p.ldc & 3) == 0) {
            red_add_v4(dst, v.x, v.y, v.z, v.w);
          } else {
            const float* vv = &v.x;
            for (int u = 0; u < 4 && col + u < p.N; ++u) atomicAdd(dst + u, vv[u]);
          }
          continue;
        }
        if (vec_ok && col + 4 <= p.N && (p.ldc & 3) == 0) {
          if (acc) {
            v.x += old[it].x; v.y += old[it].y; v.z += old[it].z; v.w += old[it].w;
          }
          *reinterpret_cast<float4*>(dst) = v;
        } else {
          const float* vv = &v.x;
          for (int u = 0; u < 4 && col + u < p.N; ++u) dst[u] = vv[u] + (acc ? dst[u] : 0.f);
        }
      }
    } else {
      __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.C);
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int row = it * 4 + (lane >> 3), c8 = lane & 7;
        const long m = m0 + row;
        const int col = cg + c8 * 8;
        if (m >= m_end || col >= p.N) continue;
        const float4 a = *reinterpret_cast<const float4*>(stage + row * 64 + (((2 * c8) ^ (row & 15)) * 4));
        const float4 b = *reinterpret_cast<const float4*>(stage + row * 64 + (((2 * c8 + 1) ^ (row & 15)) * 4));
        float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        __nv_bfloat16* dst = C + m * p.ldc + col;
        if (vec_ok && col + 8 <= p.N) {
          if (acc) {
            const uint4 o4 = *reinterpret_cast<const uint4*>(&old[it]);
            v[0] += bf16_lo(o4.x); v[1] += bf16_hi(o4.x);
            v[2] += bf16_lo(o4.y); v[3] += bf16_hi(o4.y);
            v[4] += bf16_lo(o4.z); v[5] += bf16_hi(o4.z);
            v[6] += bf16_lo(o4.w); v[7] += bf16_hi(o4.w);
          }
          uint4 o;
          o.x = pack_bf16x2(v[0], v[1]);
          o.y = pack_bf16x2(v[2], v[3]);
          o.z = pack_bf16x2(v[4], v[5]);
          o.w = pack_bf16x2(v[6], v[7]);
          *reinterpret_cast<uint4*>(dst) = o;
        } else {
          for (int u = 0; u < 8 && col + u < p.N; ++u)
            dst[u] = __float2bfloat16(v[u] + (acc ? __bfloat162float(dst[u]) : 0.f));
        }
      }
    }
    __syncwarp();
  }
}

template <int GM>
__device__ __forceinline__ TileInfo tile_info(const GemmParams& p, int tile, int num_m, int num_n, int num_kb,
                                              int BM, int BK) {
  TileInfo t{};
  if constexpr (GM == 2) {
    const int per = num_m * num_n;
    t.group = tile / per;
    tile_coords(tile - t.group * per, num_m, num_n, t.mb, t.nb);
    const int r0 = __ldg(p.offsets + t.group), r1 = __ldg(p.offsets + t.group + 1);
    t.kb0 = r0 / BK;
    t.nkb = (r1 - r0) / BK;
  } else if (GM == 0 && p.splits > 1) {
    // Slice-major order: the first wave runs slice 0 of consecutive tiles, as without a split.
    const int per = num_m * num_n;
    t.slice = tile / per;
    tile_coords(tile - t.slice * per, num_m, num_n, t.mb, t.nb);
    const int kper = (num_kb + p.splits - 1) / p.splits;
    t.kb0 = t.slice * kper;
    t.nkb = min(kper, num_kb - t.kb0);
  } else {
    tile_coords(tile, num_m, num_n, t.mb, t.nb);
    t.group = GM == 1 ? group_of_row(p.offsets, p.groups, t.mb * BM) : 0;
    t.kb0 = 0;
    t.nkb = num_kb;
  }
  return t;
}

template <int BN, bool A_MN, bool B_MN, int GM = 0>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int BM = Cfg::BM, BK = Cfg::BK, STAGES = Cfg::STAGES;
  constexpr int A_BYTES = Cfg::A_BYTES, B_BYTES = Cfg::B_BYTES;
  constexpr uint32_t IDESC = make_idesc_f16(BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* stage_base = sB + STAGES * B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_base + Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM, num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n * (GM == 2 ? p.groups : (GM == 0 && p.splits > 1 ? p.splits : 1));
  const int num_kb = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
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
      uint32_t filled_mask = 0;
      uint32_t last_phase[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_phase[s] = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const TileInfo ti = tile_info<GM>(p, tile, num_m, num_n, num_kb, BM, BK);
        const int mb = ti.mb, nb = ti.nb;
        // Mode 1: the expert's slice of the stacked B starts at group * b_group_rows rows.
        const int b_row0 = GM == 1 ? ti.group * p.b_group_rows : 0;
        for (int kq = 0; kq < ti.nkb; ++kq) {
          const int kb = ti.kb0 + kq;
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          if constexpr (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * BK, mb * BM);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * 8192, &tmA, &full[stage], mb * BM + j * 64, kb * BK);
          }
          if constexpr (!B_MN) {
            tma_load_2d(b_dst, &tmB, &full[stage], kb * BK, b_row0 + nb * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(b_dst + j * 8192, &tmB, &full[stage], nb * BN + j * 64, b_row0 + kb * BK);
          }
          filled_mask |= 1u << stage;
          last_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Never leave the CTA with a TMA write still landing in shared memory.
      for (int s = 0; s < STAGES; ++s)
        if (filled_mask & (1u << s)) mbar_wait(&full[s], last_phase[s], nullptr, 0) || true;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int tile_nkb =
            (GM == 2 || (GM == 0 && p.splits > 1)) ? tile_info<GM>(p, tile, num_m, num_n, num_kb, BM, BK).nkb : num_kb;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < tile_nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major: advance 16 elements (32 B) inside the 128 B swizzle row.
            // MN-major: advance 16 K-rows (16 x 128 B) = two 8-row swizzle atoms.
            const uint64_t adesc = A_MN ? make_smem_desc_sw128(a_base + k * 2048, 8192, 1024)
                                        : make_smem_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_smem_desc_sw128(b_base + k * 2048, 8192, 1024)
                                        : make_smem_desc_sw128(b_base + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, adesc, bdesc, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // Make sure every MMA this thread issued has retired before TMEM is freed.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    // Epilogue: warps 2..5 -> TMEM lane quarter (warp % 4).
    const int q = warp & 3;
    const int row = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool vec_ok = ((p.ldc & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
    float* stage = reinterpret_cast<float*>(stage_base + q * 8192);
    (void)row;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const TileInfo ti = tile_info<GM>(p, tile, num_m, num_n, num_kb, BM, BK);
      if (!mbar_wait(&tfull[acc], acc_phase, p.status, kStatusTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (GM != 2) {
        epilogue_tile<BN>(t_row, stage, p, static_cast<long>(ti.mb) * BM + q * 32, ti.nb * BN, vec_ok, p.M,
                          GM == 0 && p.splits > 1);
      } else if (ti.nkb > 0) {
        // Expert block: rows [group * M, group * M + M) of the stacked output; an expert without
        // rows contributes nothing (its accumulator was never written).
        const long base = static_cast<long>(ti.group) * (p.c_group_stride > 0 ? p.c_group_stride : p.M);
        epilogue_tile<BN>(t_row, stage, p, base + static_cast<long>(ti.mb) * BM + q * 32, ti.nb * BN, vec_ok,
                          base + p.M);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  if (p.pub_n > 0 && warp >= 2) __threadfence();  // this thread's C stores, before the CTA's arrival
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  if (p.pub_n > 0 && threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(p.pub_ctr, 1u);
    if (prev == gridDim.x - 1) {
      // Every CTA has arrived: their fenced stores are ordered before this point.
      __threadfence_system();
      for (int d = 0; d < p.pub_n && d < 8; ++d) st_relaxed_sys_u64(p.pub_flag[d], p.pub_epoch);
      *p.pub_ctr = 0u;  // at rest again for the next launch (kernel boundary orders it)
    }
  }
}

// ------------------------------------------------------------------ CTA-pair (2-SM) GEMM
// Plain GEMM on 256 x 256 tiles computed by a cluster of two CTAs on two SMs. CTA r of the pair
// loads rows [128 r, 128 r + 128) of the tile's A and columns [128 r, 128 r + 128) of its B into its
// own shared memory (no multicast), both loads completing on CTA 0's `full` barrier; CTA 0's MMA
// warp issues tcgen05.mma.cta_group::2 (M = 256, N = 256), which reads both CTAs' operands and
// writes rows [128 r, 128 r + 128) of the accumulator into CTA r's TMEM, and commits to the
// `empty` / `tfull` barriers of both CTAs. Each CTA's epilogue drains its own half and arrives on
// CTA 0's `tempty`. Per SM and K block, the tile moves 32 KB from L2 instead of the 48 KB of a
// 128 x 256 single-CTA tile, for the same tensor-core work, and the six-stage ring fits.
// Same parameters (fp32 accumulate, K slices, publication) as gemm_bf16_kernel with GM = 0.
struct PairCfg {
  static constexpr int BM = 128;  // rows per CTA; the pair covers 256
  static constexpr int BN = 256;  // columns of the pair tile; each CTA holds 128 of B
  static constexpr int BK = 64;
  static constexpr int STAGES = 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int STAGE_BYTES = 4 * 8192;
  static constexpr int SMEM_BYTES = 1024 + STAGES * (A_BYTES + B_BYTES) + STAGE_BYTES + 256;
};

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          GemmParams p) {
  using Cfg = PairCfg;
  constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, STAGES = Cfg::STAGES;
  constexpr int A_BYTES = Cfg::A_BYTES, B_BYTES = Cfg::B_BYTES;
  constexpr uint32_t IDESC = make_idesc_f16(2 * BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* stage_base = sB + STAGES * B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_base + Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int num_m = (p.M + 2 * BM - 1) / (2 * BM), num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n * (p.splits > 1 ? p.splits : 1);
  const int num_kb = (p.K + BK - 1) / BK;
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * 128);  // every epilogue thread of both CTAs
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before either CTA signals the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full0 = cluster_addr(full, 0);      // CTA 0's full[s] at full0 + 8 s
  const uint32_t tempty0 = cluster_addr(tempty, 0);  // CTA 0's tempty[b] at tempty0 + 8 b

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t filled_mask = 0;
      uint32_t last_phase[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_phase[s] = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        const TileInfo ti = tile_info<0>(p, tile, num_m, num_n, num_kb, 2 * BM, BK);
        const int arow = ti.mb * 2 * BM + static_cast<int>(rank) * BM;
        const int bcol = ti.nb * BN + static_cast<int>(rank) * (BN / 2);
        for (int kq = 0; kq < ti.nkb; ++kq) {
          const int kb = ti.kb0 + kq;
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          // CTA 0 expects the bytes of both CTAs' loads on its barrier.
          if (rank == 0) mbar_expect_tx(&full[stage], 2 * (A_BYTES + B_BYTES));
          const uint32_t bar = full0 + 8u * static_cast<uint32_t>(stage);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          if constexpr (!A_MN) {
            tma_load_2d_pair(a_dst, &tmA, bar, kb * BK, arow);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d_pair(a_dst + j * 8192, &tmA, bar, arow + j * 64, kb * BK);
          }
          if constexpr (!B_MN) {
            tma_load_2d_pair(b_dst, &tmB, bar, kb * BK, bcol);
          } else {
#pragma unroll
            for (int j = 0; j < (BN / 2) / 64; ++j)
              tma_load_2d_pair(b_dst + j * 8192, &tmB, bar, bcol + j * 64, kb * BK);
          }
          filled_mask |= 1u << stage;
          last_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // CTA 0's barriers count both CTAs' bytes: never leave with a TMA write still landing.
      if (rank == 0)
        for (int s = 0; s < STAGES; ++s)
          if (filled_mask & (1u << s)) mbar_wait(&full[s], last_phase[s], nullptr, 0) || true;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        const int tile_nkb = p.splits > 1 ? tile_info<0>(p, tile, num_m, num_n, num_kb, 2 * BM, BK).nkb : num_kb;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < tile_nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? make_smem_desc_sw128(a_base + k * 2048, 8192, 1024)
                                        : make_smem_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_smem_desc_sw128(b_base + k * 2048, 8192, 1024)
                                        : make_smem_desc_sw128(b_base + k * 32, 16, 1024);
            umma_f16_ss_pair(d_tmem, adesc, bdesc, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(cluster_addr(&empty[stage], 0));
          umma_commit_pair(cluster_addr(&empty[stage], 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(cluster_addr(&tfull[acc], 0));
        umma_commit_pair(cluster_addr(&tfull[acc], 1));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // Every MMA (which reads both CTAs' shared memory) retires before either CTA moves on.
      umma_commit_pair(cluster_addr(drain, 0));
      mbar_wait(drain, 0, nullptr, 0);
    }
  } else {
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool vec_ok = ((p.ldc & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
    float* stage = reinterpret_cast<float*>(stage_base + q * 8192);
    for (int tile = pair; tile < num_tiles; tile += npairs) {
      const TileInfo ti = tile_info<0>(p, tile, num_m, num_n, num_kb, 2 * BM, BK);
      if (!mbar_wait(&tfull[acc], acc_phase, p.status, kStatusTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      epilogue_tile<BN>(t_row, stage, p, static_cast<long>(ti.mb) * 2 * BM + rank * BM + q * 32, ti.nb * BN,
                        vec_ok, p.M, p.splits > 1);
      tc_fence_before();
      mbar_arrive_cluster(tempty0 + 8u * static_cast<uint32_t>(acc));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  if (p.pub_n > 0 && warp >= 2) __threadfence();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // CTA 0's MMAs have retired and every cross-CTA arrival has landed
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
  if (p.pub_n > 0 && threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(p.pub_ctr, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < p.pub_n && d < 8; ++d) st_relaxed_sys_u64(p.pub_flag[d], p.pub_epoch);
      *p.pub_ctr = 0u;
    }
  }
}

// ------------------------------------------------------------------ host side

template <int BN, bool A_MN, bool B_MN, int GM = 0>
static void launch_gemm(const CUtensorMap* ta, const CUtensorMap* tb, GemmParams p, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_bf16_kernel<BN, A_MN, B_MN, GM>;
  static bool attr_set[16] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 15]) {
    NTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    attr_set[dev & 15] = true;
  }
  const int num_tiles = ((p.M + Cfg::BM - 1) / Cfg::BM) * ((p.N + BN - 1) / BN) *
                        (GM == 2 ? p.groups : (GM == 0 && p.splits > 1 ? p.splits : 1));
  const int grid = std::min(num_tiles, num_sms(dev));
  void* args[3] = {const_cast<CUtensorMap*>(ta), const_cast<CUtensorMap*>(tb), &p};
  NTB_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(192), args,
                                  Cfg::SMEM_BYTES, stream));
  NTB_LAUNCH_CHECK(1);
}

template <bool A_MN, bool B_MN>
static void launch_gemm_pair(const CUtensorMap* ta, const CUtensorMap* tb, GemmParams p, cudaStream_t stream) {
  auto kern = gemm_bf16_pair_kernel<A_MN, B_MN>;
  static bool attr_set[16] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 15]) {
    NTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg::SMEM_BYTES));
    attr_set[dev & 15] = true;
  }
  const int units = ((p.M + 2 * PairCfg::BM - 1) / (2 * PairCfg::BM)) * ((p.N + PairCfg::BN - 1) / PairCfg::BN) *
                    (p.splits > 1 ? p.splits : 1);
  const int pairs = std::max(1, std::min(units, num_sms(dev) / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = PairCfg::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[3] = {const_cast<CUtensorMap*>(ta), const_cast<CUtensorMap*>(tb), &p};
  NTB_CUDA_CHECK(cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(kern), args));
  NTB_LAUNCH_CHECK(1);
}

// Tile shape of a dense GEMM: the tile width (128 or 256) and, for an fp32 accumulated
// C without bias (weight gradients into fp32 main grads), a split of K into 1-3 slices.
// Every unit of the persistent kernel runs the same K loop, so the kernel's time is
// (waves of units) x (time of one unit). Measured on B200 (bench/profile_kernels.py gemm):
//   - a 128-wide tile runs at about 0.63 of the 256-wide tile's rate (4096^3: 155.6 us
//     against 112.6 us for 7 waves of narrow against 4 waves of wide tiles), so it wins
//     only where the wide tiles leave most SMs idle;
//   - a K slice adds its partial to C with fire-and-forget vector reductions; fitted over
//     768..6144 x 512..4096 x 4096 weight gradients, two slices cost 6.5 % and three 29 % on
//     top of the wave count (1.07x faster at 4096^3 and 3584 x 4096 with two slices, 1.2x at
//     768 x 4096 with three, 0.84x at 4096^3 with three), so a split is taken only where the
//     model saves more than 5 %.
// Tensor-parallel ranks gain most: an N = 512 weight gradient is 64 wide tiles on 148 SMs.
// NTB_GEMM_BN=128|256 forces the width; NTB_GEMM_SPLITK=0 turns the split off, =2..4 forces it.
struct TileChoice {
  bool wide;
  int splits;
};

static TileChoice pick_tiles(int64_t M, int64_t N, int64_t K, int nsm, bool can_split) {
  static const int forced_bn = [] {
    const char* e = std::getenv("NTB_GEMM_BN");
    return e ? std::atoi(e) : 0;
  }();
  static const int forced_split = [] {  // -1: automatic, 0: off, 2..4: that many slices where allowed
    const char* e = std::getenv("NTB_GEMM_SPLITK");
    return e ? std::atoi(e) : -1;
  }();
  constexpr double kNarrowRate = 0.63;     // rate of a 128-wide tile relative to a 256-wide one
  constexpr double kSliceCost[4] = {1.0, 1.0, 1.065, 1.29};  // time factor of a unit split into s slices
  constexpr double kSplitMargin = 0.95;    // a split must beat the best unsplit shape by 5 %
  constexpr int64_t kMinSliceBlocks = 16;  // K blocks of 64 per slice, so the pipeline stays full
  const int64_t mt = (M + 127) / 128, kb = (K + 63) / 64;
  auto cost = [&](bool wide, int sp) {
    const int64_t units = mt * ((N + (wide ? 255 : 127)) / (wide ? 256 : 128)) * sp;
    const double w = static_cast<double>((units + nsm - 1) / nsm);
    return w / sp * (wide ? 1.0 : 0.5 / kNarrowRate) * kSliceCost[sp];
  };
  auto width_ok = [&](bool wide) {
    if (wide && N <= 128) return false;
    if (forced_bn == 128) return !wide;
    if (forced_bn == 256) return wide || N <= 128;
    return true;
  };
  TileChoice best{N > 128, 1};
  double best_cost = 1e30;
  for (int w = 1; w >= 0; --w)
    if (width_ok(w == 1) && cost(w == 1, 1) < best_cost - 1e-9) {
      best_cost = cost(w == 1, 1);
      best = {w == 1, 1};
    }
  if (!can_split || forced_split == 0) return best;
  if (forced_split >= 2) {
    const int sp = static_cast<int>(std::min<int64_t>(forced_split, std::max<int64_t>(1, kb / kMinSliceBlocks)));
    return {best.wide, std::min(sp, 4)};
  }
  const double bar = best_cost * kSplitMargin;
  TileChoice split = best;
  double split_cost = 1e30;
  for (int w = 1; w >= 0; --w) {
    if (!width_ok(w == 1)) continue;
    for (int sp = 2; sp <= 3 && kb >= kMinSliceBlocks * sp; ++sp)
      if (cost(w == 1, sp) < split_cost - 1e-9) {
        split_cost = cost(w == 1, sp);
        split = {w == 1, sp};
      }
  }
  return split_cost < bar ? split : best;
}

// Builds the TMA descriptor of one operand. K-major operands are read as
// [rows, K] boxes of 64 x rows_box; MN-major operands as [K, MN] boxes of
// 64 x 64 (the swizzled K-row is the 64-element MN strip).
static void operand_map(CUtensorMap* out, const at::Tensor& t, bool mn_major, int rows_box) {
  const int64_t d0 = t.size(1), d1 = t.size(0);
  const int64_t ld = t.stride(0);
  make_tma_2d_bf16(out, t.data_ptr(), d0, d1, ld, 64, mn_major ? 64 : rows_box);
}

// out = alpha * op(a) . op(b)^T (+ bias) (+ out if accumulate).
//   a: [M,K] (a_mn=false) or [K,M] (a_mn=true), bf16, unit inner stride
//   b: [N,K] (b_mn=false) or [K,N] (b_mn=true), bf16, unit inner stride
//   out: [M,N] bf16 or fp32 with unit inner stride
static void gemm_bf16_impl(const at::Tensor& a, const at::Tensor& b, at::Tensor& out,
                           const c10::optional<at::Tensor>& bias, bool a_mn, bool b_mn, bool accumulate, double alpha,
                           const std::vector<int64_t>& pub_flags, int64_t pub_epoch, unsigned int* pub_ctr) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "gemm_bf16: CUDA tensors required");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_bf16: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm_bf16: 2-D tensors");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1, "gemm_bf16: inner stride must be 1");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat, "gemm_bf16: bf16/fp32 out");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm_bf16: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm_bf16: bad out shape");
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0, "gemm_bf16: row stride must be 16B aligned");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(a.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(b.data_ptr()) & 15) == 0,
              "gemm_bf16: operands must be 16B aligned");
  // A publishing launch must run (peers wait for its epoch).
  TORCH_CHECK(pub_flags.empty() || (M > 0 && N > 0 && K > 0), "gemm_bf16_publish: empty problem");
  if (M == 0 || N == 0) return;
  if (K == 0) {
    if (!accumulate) out.zero_();
    if (bias.has_value()) out.add_(bias.value());
    return;
  }
  GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = out.data_ptr();
  p.ldc = out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias.value().data_ptr()) : nullptr;
  if (bias.has_value()) TORCH_CHECK(bias.value().scalar_type() == at::kBFloat16 && bias.value().numel() == N, "gemm_bf16: bias");
  p.alpha = static_cast<float>(alpha);
  p.accumulate = accumulate ? 1 : 0;
  p.c_f32 = out.scalar_type() == at::kFloat ? 1 : 0;
  p.status = device_status(a.get_device());
  p.offsets = nullptr;
  p.groups = 1;
  p.b_group_rows = 0;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(a.get_device());
  const TileChoice tc = pick_tiles(M, N, K, num_sms(a.get_device()),
                                   accumulate && p.c_f32 && !bias.has_value());
  const bool wide = tc.wide;
  p.splits = tc.splits;
  if (!pub_flags.empty()) {
    TORCH_CHECK(pub_flags.size() <= 8 && pub_ctr != nullptr && !accumulate, "gemm_bf16: publication to 1..8 flags");
    for (size_t i = 0; i < pub_flags.size(); ++i) p.pub_flag[i] = reinterpret_cast<unsigned long long*>(pub_flags[i]);
    p.pub_n = static_cast<int>(pub_flags.size());
    p.pub_epoch = static_cast<unsigned long long>(pub_epoch);
    p.pub_ctr = pub_ctr;
    p.splits = 1;
  }
  // CTA-pair tiles (256 x 256 on two SMs): measured 3-7 % faster than the single-CTA 128 x 256
  // tile once each unit runs at least 2048 of K (4096^3: 107.5 against 113.7 us; 4096 x 4096 x
  // 14336: 338.9 against 361.5 us; 4096^3 weight gradient in two K slices: 108.6 against 114.7 us)
  // and up to 10 % slower on short K (K = 512: 44.0 against 39.9 us), where the pair's extra
  // prologue is not amortised. NTB_GEMM_2SM=0 turns them off, =1 uses them for every wide tile.
  static const int pair_mode = [] {
    const char* e = std::getenv("NTB_GEMM_2SM");
    return e ? std::atoi(e) : -1;
  }();
  const bool pair = wide && M >= 256 && pair_mode != 0 && (pair_mode == 1 || K / std::max(1, tc.splits) >= 2048);
  TmaSlots& slots = tls_tma_slots();
  CUtensorMap* ta = &slots.m[0];
  CUtensorMap* tb = &slots.m[1];
  operand_map(ta, a, a_mn, 128);
  operand_map(tb, b, b_mn, (wide && !pair) ? 256 : 128);
  if (pair) {
    if (!a_mn && !b_mn) launch_gemm_pair<false, false>(ta, tb, p, stream);
    else if (!a_mn && b_mn) launch_gemm_pair<false, true>(ta, tb, p, stream);
    else if (a_mn && !b_mn) launch_gemm_pair<true, false>(ta, tb, p, stream);
    else launch_gemm_pair<true, true>(ta, tb, p, stream);
    return;
  }
#define NTB_GEMM_CASE(BN_, AM, BM_)                     \
  if (a_mn == AM && b_mn == BM_) {                      \
    launch_gemm<BN_, AM, BM_>(ta, tb, p, stream);       \
    return;                                             \
  }
  if (wide) {
    NTB_GEMM_CASE(256, false, false) NTB_GEMM_CASE(256, false, true) NTB_GEMM_CASE(256, true, false)
    NTB_GEMM_CASE(256, true, true)
  } else {
    NTB_GEMM_CASE(128, false, false) NTB_GEMM_CASE(128, false, true) NTB_GEMM_CASE(128, true, false)
    NTB_GEMM_CASE(128, true, true)
  }
#undef NTB_GEMM_CASE
}

void gemm_bf16(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, const c10::optional<at::Tensor>& bias,
               bool a_mn, bool b_mn, bool accumulate, double alpha) {
  gemm_bf16_impl(a, b, out, bias, a_mn, b_mn, accumulate, alpha, {}, 0, nullptr);
}

// out = a . op(b)^T, then the last CTA publishes `epoch` to every address of `flags` (device
// u64 epoch words, typically the peers' copies of this rank's flag) after a system-scope fence,
// so peers may read `out` over NVLink once they see the epoch. `ctr`: int32 device word, zero.
void gemm_bf16_publish(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, bool b_mn,
                       std::vector<int64_t> flags, int64_t epoch, at::Tensor& ctr) {
  TORCH_CHECK(ctr.is_cuda() && ctr.scalar_type() == at::kInt && ctr.numel() >= 1, "gemm_bf16_publish: int32 ctr");
  TORCH_CHECK(!flags.empty(), "gemm_bf16_publish: at least one flag");
  gemm_bf16_impl(a, b, out, c10::nullopt, false, b_mn, false, 1.0, flags, epoch,
                 reinterpret_cast<unsigned int*>(ctr.data_ptr()));
}

// Grouped GEMM for mixture-of-experts layers. `offsets` (int32 [G + 1], device) are the
// row offsets of the G expert segments of the token-major operands; every offset must
// be a multiple of 128 (segments are padded with zero rows).
//   mode 1 (M-grouped): out[rows of g] = a[rows of g] . op(B_g)^T
//        a: [R, K] tokens;  b: stacked [G * N, K] (b_mn=false, forward)
//                              or [G * K, N] (b_mn=true, input gradient);  out: [R, N]
//   mode 2 (K-grouped): out[g] (+)= a[rows of g]^T . b[rows of g]
//        a: [R, M] (e.g. dY), b: [R, N] (e.g. X), out: stacked [G * M, N] (fp32 weight gradient)
void gemm_grouped_bf16(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, const at::Tensor& offsets,
                       int64_t mode, bool b_mn, bool accumulate, int64_t c_group_stride) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda() && offsets.is_cuda(), "gemm_grouped: CUDA tensors");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_grouped: bf16 operands");
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.dim() == 1 && offsets.numel() >= 2 &&
                  offsets.is_contiguous(),
              "gemm_grouped: int32 offsets [G + 1]");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 &&
                  out.stride(1) == 1,
              "gemm_grouped: 2-D tensors with unit inner stride");
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0, "gemm_grouped: 16-byte row strides");
  const int G = static_cast<int>(offsets.numel() - 1);
  GemmParams p{};
  p.offsets = offsets.data_ptr<int>();
  p.groups = G;
  p.alpha = 1.f;
  p.accumulate = accumulate ? 1 : 0;
  p.c_f32 = out.scalar_type() == at::kFloat ? 1 : 0;
  p.C = out.data_ptr();
  p.ldc = out.stride(0);
  p.bias = nullptr;
  p.status = device_status(a.get_device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(a.get_device());
  TmaSlots& slots = tls_tma_slots();
  if (mode == 1) {
    TORCH_CHECK(b.size(0) % G == 0, "gemm_grouped: stacked B rows must divide by the group count");
    const int64_t R = a.size(0), K = a.size(1);
    const int64_t rows_g = b.size(0) / G;
    const int64_t N = b_mn ? b.size(1) : rows_g;
    TORCH_CHECK((b_mn ? rows_g : b.size(1)) == K, "gemm_grouped: K mismatch");
    TORCH_CHECK(out.size(0) == R && out.size(1) == N, "gemm_grouped: out shape");
    TORCH_CHECK(R % 128 == 0, "gemm_grouped: rows must be padded to a multiple of 128");
    if (R == 0 || N == 0) return;
    p.M = static_cast<int>(R);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.b_group_rows = static_cast<int>(rows_g);
    const bool wide = N > 128;
    operand_map(&slots.m[0], a, false, 128);
    operand_map(&slots.m[1], b, b_mn, wide ? 256 : 128);
    if (wide) {
      if (b_mn) launch_gemm<256, false, true, 1>(&slots.m[0], &slots.m[1], p, stream);
      else launch_gemm<256, false, false, 1>(&slots.m[0], &slots.m[1], p, stream);
    } else {
      if (b_mn) launch_gemm<128, false, true, 1>(&slots.m[0], &slots.m[1], p, stream);
      else launch_gemm<128, false, false, 1>(&slots.m[0], &slots.m[1], p, stream);
    }
    return;
  }
  TORCH_CHECK(mode == 2, "gemm_grouped: mode 1 or 2");
  TORCH_CHECK(a.size(0) == b.size(0), "gemm_grouped: a and b must have the same rows");
  const int64_t M = a.size(1), N = b.size(1);
  if (c_group_stride > 0) {
    // Group g's [M, N] block starts at row g * c_group_stride of out (e.g. per-expert gradients inside a
    // flat buffer that interleaves other parameters between the experts' blocks).
    TORCH_CHECK(c_group_stride >= M && out.size(1) == N && out.size(0) >= (G - 1) * c_group_stride + M,
                "gemm_grouped: out must hold (G - 1) * c_group_stride + M rows of N");
    p.c_group_stride = c_group_stride;
  } else {
    TORCH_CHECK(out.size(0) == G * M && out.size(1) == N, "gemm_grouped: out must be [G * M, N]");
  }
  if (M == 0 || N == 0) return;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(a.size(0));
  const bool wide = N > 128;
  operand_map(&slots.m[0], a, true, 128);
  operand_map(&slots.m[1], b, true, wide ? 256 : 128);
  if (wide) launch_gemm<256, true, true, 2>(&slots.m[0], &slots.m[1], p, stream);
  else launch_gemm<128, true, true, 2>(&slots.m[0], &slots.m[1], p, stream);
}

}  // namespace ntb
