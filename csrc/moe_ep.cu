// Expert-parallel MoE dispatch and combine over NVLink peer memory.
//
// Every rank of the expert-parallel group owns one symmetric workspace (CUDA
// IPC, same layout everywhere) holding, per source rank, a slab of received
// rows (payload bf16, or e4m3 + one fp32 scale per 128 columns) with a 16-byte
// record {local expert, source token, routing weight, top-k slot} per row, a
// row map (slab row -> row of the expert-grouped GEMM input, -1 if dropped by
// capacity), the expert outputs, the gradient of the expert inputs, the
// gradient of this rank's MoE output, and flag words.
//
// Forward
//   ep_dispatch  (sender, ONE launch): each warp takes assignments in
//                destination-sorted order and stores the token row straight
//                into the destination's slab (peer stores over NVLink),
//                quantising to e4m3 with 1x128 scales on the way when the
//                payload is fp8 (same numerics as the tile quantiser, the
//                random bits of stochastic rounding indexed by the sorted
//                payload element). The last CTA to finish writes the row
//                count and token count into every destination's info words
//                and publishes the epoch in its flag (system-scope release).
//   ep_wait      bounded wait until every source's flag shows the epoch.
//   ep_gather    (receiver, local): capacity-selected rows of the slab ->
//                the zero-padded, expert-grouped GEMM input (dequantised).
//   grouped GEMMs write the expert outputs into the workspace; ep_signal.
//   ep_pull      (sender, ONE launch): one warp per token reads the row map
//                and the K expert-output rows of that token from the peers
//                (peer loads), and writes sum_k w_k * y_k: the combine and its
//                weighted reduction in one pass. It keeps the pulled rows and
//                their positions for the backward.
// Backward
//   ep_combine_bwd (receiver): dY row = w * dOut[token] read from the
//                source's workspace (peer loads), zero for padding rows.
//   ep_pull      again with unit weights over the expert-input gradients: the
//                dispatch backward (sum over the K copies of each token).
//
// Every wait is bounded (status word), every index read from another rank's
// memory is range-checked before it addresses anything.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "fp8_util.cuh"
#include "host_utils.h"
#include "peer.cuh"

#include <vector>

namespace ntb {
namespace {

using bf16 = __nv_bfloat16;
constexpr int kEpMaxRanks = 8;
constexpr int kEpMaxTopK = 8;
constexpr int kWarps = 8;  // 256-thread CTAs, one row per warp at a time

__device__ __forceinline__ void unpack_bf16x8(const uint4& r, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&v)[8]) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
  return r;
}

// amax over the 16 lanes of a half warp (one 128-column tile at 8 columns per lane).
__device__ __forceinline__ float half_warp_max(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Quantises 8 consecutive values (columns c..c+7 of payload row `row`) to e4m3
// with scale s, exactly as the tile quantiser: y = clamp(v / s), optional
// stochastic rounding keyed by the element index row * H + c + j.
__device__ __forceinline__ uint2 quant8(const float (&v)[8], float s, bool stochastic, uint64_t seed,
                                        uint64_t elem0) {
  uint32_t w[2] = {0u, 0u};
  const ScaleDiv sd = make_scale_div(s);  // the correctly rounded v / s, as the tile quantiser
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float y = fminf(fmaxf(div_scale(v[j], sd), -448.f), 448.f);
    if (stochastic) y = e4m3_sr(y, uniform01(seed, elem0 + j));
    w[j >> 2] |= static_cast<uint32_t>(to_e4m3(y)) << (8 * (j & 3));
  }
  return make_uint2(w[0], w[1]);
}

// Dequantised row chunk rounded to bf16 (the dtype the unfused path carries).
__device__ __forceinline__ void dequant8(const uint2& q, float s, float (&v)[8]) {
  const uint32_t w[2] = {q.x, q.y};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float f = from_e4m3(static_cast<uint8_t>(w[j >> 2] >> (8 * (j & 3)))) * s;
    v[j] = __bfloat162float(__float2bfloat16(f));
  }
}

// ------------------------------------------------------------------ dispatch
struct EpDispatchParams {
  const bf16* x;              // [T, H] this rank's tokens
  long H;
  int T, K, epr;
  const int64_t* idx;         // [T, K] global expert of each assignment (router output)
  const void* w;              // [T, K] routing weight (bf16 or fp32)
  int w_f32;
  int* dest_tk;               // out [T*K] destination rank of assignment (t, k)
  int* slot_tk;               // out [T*K] row in this source's block of the destination slab
  int* ctr;                   // [n] local slot counters (zero at rest)
  uint8_t* payload[kEpMaxRanks];  // destination slab payload, this source's block already applied
  float* pscale[kEpMaxRanks];     // fp8 payload scales (same block)
  int4* meta[kEpMaxRanks];        // per-row records (same block)
  unsigned long long* flag[kEpMaxRanks];  // destination's dispatch flag for this source
  int* info[kEpMaxRanks];                 // destination's info words for this source
  long P;  // slab rows per source
  int n;
  int fp8, stochastic;
  unsigned long long seed;
  unsigned int* done;  // local arrival counter (zero at rest)
  unsigned long long epoch;
  int* status;
};

// One warp per (token, k) assignment in token order. Lane 0 reserves the next
// row of this source's block in the destination slab (atomic on a local
// counter), so no sort precedes the exchange; the receiver orders rows by a
// total key, which makes the result independent of the reservation order.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const EpDispatchParams p) {
  const int lane = threadIdx.x & 31;
  const long nwarps = static_cast<long>(gridDim.x) * kWarps;
  const long n_assign = static_cast<long>(p.T) * p.K;
  for (long a = static_cast<long>(blockIdx.x) * kWarps + (threadIdx.x >> 5); a < n_assign; a += nwarps) {
    const int t = static_cast<int>(a / p.K), k = static_cast<int>(a % p.K);
    const long e = __ldg(p.idx + a);
    const int d = static_cast<int>(e / p.epr);
    if (e < 0 || d >= p.n) {
      if (lane == 0) {
        set_status(p.status, kStatusBadShape);
        p.dest_tk[a] = 0;
        p.slot_tk[a] = -1;
      }
      continue;
    }
    int s = 0;
    if (lane == 0) s = atomicAdd(p.ctr + d, 1);
    s = __shfl_sync(0xffffffffu, s, 0);
    if (s >= p.P) {  // cannot happen for T*K <= P; never write past the block
      if (lane == 0) {
        set_status(p.status, kStatusBadShape);
        p.dest_tk[a] = d;
        p.slot_tk[a] = -1;
      }
      continue;
    }
    const bf16* src = p.x + static_cast<long>(t) * p.H;
    if (!p.fp8) {
      bf16* dst = reinterpret_cast<bf16*>(p.payload[d]) + static_cast<long>(s) * p.H;
#pragma unroll 4
      for (long c = lane * 8; c < p.H; c += 256)
        *reinterpret_cast<uint4*>(dst + c) = __ldg(reinterpret_cast<const uint4*>(src + c));
    } else {
      uint8_t* dst = p.payload[d] + static_cast<long>(s) * p.H;
      float* sc = p.pscale[d] + static_cast<long>(s) * (p.H / 128);
      for (long c0 = 0; c0 < p.H; c0 += 256) {
        const long c = c0 + lane * 8;
        const bool act = c < p.H;  // uniform per half warp (H % 128 == 0)
        float v[8];
        float amax = 0.f;
        if (act) {
          unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(src + c)), v);
#pragma unroll
          for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
        }
        amax = half_warp_max(amax);
        const float scale = amax > 0.f ? amax / 448.f : 1.f;
        if (act) {
          *reinterpret_cast<uint2*>(dst + c) =
              quant8(v, scale, p.stochastic != 0, p.seed, static_cast<uint64_t>(a) * p.H + c);
          if ((lane & 15) == 0) sc[c / 128] = scale;
        }
      }
    }
    if (lane == 0) {
      const float wv = p.w_f32 ? reinterpret_cast<const float*>(p.w)[a]
                               : __bfloat162float(reinterpret_cast<const bf16*>(p.w)[a]);
      p.meta[d][s] = make_int4(static_cast<int>(e - static_cast<long>(d) * p.epr), t, __float_as_int(wv), k);
      p.dest_tk[a] = d;
      p.slot_tk[a] = s;
    }
  }
  // The last CTA to finish publishes: counts, then the epoch, to every destination.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < p.n; ++d) {
        p.info[d][0] = min(p.ctr[d], static_cast<int>(p.P));
        p.info[d][1] = p.T;
        p.ctr[d] = 0;
      }
      __threadfence_system();
      for (int d = 0; d < p.n; ++d) st_relaxed_sys_u64(p.flag[d], p.epoch);
      *p.done = 0u;
    }
  }
}

// ------------------------------------------------------------------ receiver: capacity selection
// Sort key of a received row (int64, ascending = keep first):
//   bits 55..62 local expert (epr for an empty slab row), 23..54 the routing weight in
//   descending order, 20..22 source rank, 0..19 the source's flat assignment t * K + k.
// The unfused module keeps, per expert, the highest weights with ties in arrival order
// (source rank, then the source's assignments in token order): the same total order.
struct EpKeyParams {
  const int4* meta;       // local slab records [n][P]
  const int* info;        // [n][4] rows received from each source
  long long* keys;        // [n * P]
  int* counts;            // [epr] rows per local expert (zeroed by the caller)
  long P;
  int n, epr, K;
};

__device__ __forceinline__ unsigned int desc_weight_key(int bits) {
  const unsigned int b = static_cast<unsigned int>(bits);
  const unsigned int asc = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return 0xFFFFFFFFu - asc;
}

__global__ void __launch_bounds__(256) ep_recv_keys_kernel(const EpKeyParams p) {
  __shared__ int s_cnt[256];
  for (int e = threadIdx.x; e < p.epr; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  const long total = static_cast<long>(p.n) * p.P;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(i / p.P);
    const long r = i - static_cast<long>(s) * p.P;
    long long key;
    if (r < min(static_cast<long>(p.info[s * 4]), p.P)) {
      const int4 m = p.meta[i];
      const int le = min(max(m.x, 0), p.epr - 1);
      const long flat = static_cast<long>(m.y) * p.K + m.w;
      key = (static_cast<long long>(le) << 55) | (static_cast<long long>(desc_weight_key(m.z)) << 23) |
            (static_cast<long long>(s) << 20) | (flat & 0xFFFFF);
      atomicAdd(&s_cnt[le], 1);
    } else {
      key = static_cast<long long>(p.epr) << 55 | (i & 0x7FFFFFFFFFFFLL);
    }
    p.keys[i] = key;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < p.epr; e += blockDim.x)
    if (s_cnt[e]) atomicAdd(p.counts + e, s_cnt[e]);
}

struct EpLayoutParams {
  const long long* skeys;  // sorted keys [n * P]
  const int64_t* order;    // original slab index of each sorted key
  const int4* meta;
  const int* info;         // for the capacity: sum of the sources' token counts
  const int* counts;       // [epr]
  int* offsets;            // out [epr + 1]
  int* row_src;            // out [rows]
  int* row_slot;
  int* row_tok;
  float* row_w;
  int* rowmap;             // out [n * P] (local symmetric memory)
  float* stats;            // out [2] dropped, received
  long P, rows;
  int n, epr, K, E;
  double capacity_factor;
  long host_cap;
};

// Prefix sums of the (capacity-clamped, 128-padded) expert counts in shared memory,
// then: kept sorted rows -> their grouped row; padding rows -> source -1.
__global__ void __launch_bounds__(256) ep_recv_layout_kernel(const EpLayoutParams p) {
  __shared__ int s_start[257], s_off[257], s_kept[256];
  __shared__ long s_cap;
  if (threadIdx.x == 0) {
    long t_all = 0;
    for (int s = 0; s < p.n; ++s) t_all += p.info[s * 4 + 1];
    double c = ceil(p.capacity_factor * static_cast<double>(t_all) * p.K / static_cast<double>(p.E));
    long cap = c < 1.0 ? 1 : static_cast<long>(c);
    s_cap = cap < p.host_cap ? cap : p.host_cap;
    int st = 0, off = 0;
    for (int e = 0; e < p.epr; ++e) {
      const int c_e = p.counts[e];
      const int kept = static_cast<int>(c_e < s_cap ? c_e : s_cap);
      s_start[e] = st;
      s_off[e] = off;
      s_kept[e] = kept;
      st += c_e;
      off += (kept + 127) / 128 * 128;
    }
    s_start[p.epr] = st;
    s_off[p.epr] = off;
    if (blockIdx.x == 0) {
      for (int e = 0; e <= p.epr; ++e) p.offsets[e] = s_off[e];
      long kept_total = 0;
      for (int e = 0; e < p.epr; ++e) kept_total += s_kept[e];
      p.stats[0] = static_cast<float>(st - kept_total);
      p.stats[1] = static_cast<float>(st);
    }
  }
  __syncthreads();
  const long valid = s_start[p.epr];
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < valid; i += stride) {
    const long long key = p.skeys[i];
    const int le = static_cast<int>(key >> 55);
    const long o = p.order[i];
    if (le >= p.epr || o < 0 || o >= static_cast<long>(p.n) * p.P) continue;
    const long r = i - s_start[le];
    if (r < s_kept[le]) {
      const long pos = s_off[le] + r;
      if (pos < p.rows) {
        const int4 m = p.meta[o];
        p.row_src[pos] = static_cast<int>(o / p.P);
        p.row_slot[pos] = static_cast<int>(o % p.P);
        p.row_tok[pos] = m.y;
        p.row_w[pos] = __int_as_float(m.z);
        p.rowmap[o] = static_cast<int>(pos);
      } else {
        p.rowmap[o] = -1;
      }
    } else {
      p.rowmap[o] = -1;
    }
  }
  // padding rows of every expert segment
  const long used = min(static_cast<long>(s_off[p.epr]), p.rows);
  for (long r = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; r < used; r += stride) {
    int lo = 0, hi = p.epr - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_off[mid] <= r) lo = mid;
      else hi = mid - 1;
    }
    if (r - s_off[lo] >= s_kept[lo]) p.row_src[r] = -1;
  }
}

// ------------------------------------------------------------------ flags
__global__ void ep_wait_kernel(const unsigned long long* flags, int n, unsigned long long epoch, int* status) {
  const int j = threadIdx.x;
  if (j < n) spin_until([&] { return ld_acquire_sys_u64(flags + j) >= epoch; }, status, kStatusTimeoutPeer);
}

struct EpSignalParams {
  unsigned long long* flag[kEpMaxRanks];
  int n;
  unsigned long long epoch;
};

// Publishes everything the preceding kernels of this stream wrote.
__global__ void ep_signal_kernel(const EpSignalParams p) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  for (int d = 0; d < p.n; ++d) st_relaxed_sys_u64(p.flag[d], p.epoch);
}

// ------------------------------------------------------------------ receiver: slab -> grouped GEMM input
struct EpGatherParams {
  const uint8_t* payload;  // local slab [n][P] rows
  const float* pscale;
  const int* rows_used;    // device: last offset (rows of the grouped layout in use)
  const int* row_src;      // [rows_cap] source rank of each grouped row, -1 = padding
  const int* row_slot;     // [rows_cap] slab row inside the source's block
  bf16* out;               // [rows_cap, H]
  long H, P, rows_cap;
  int n, fp8;
  int* status;
};

__global__ void __launch_bounds__(256) ep_gather_kernel(const EpGatherParams p) {
  const int lane = threadIdx.x & 31;
  const long rows = min(static_cast<long>(*p.rows_used), p.rows_cap);
  const long nwarps = static_cast<long>(gridDim.x) * kWarps;
  for (long r = static_cast<long>(blockIdx.x) * kWarps + (threadIdx.x >> 5); r < rows; r += nwarps) {
    const int s = __ldg(p.row_src + r);
    const int k = s >= 0 ? __ldg(p.row_slot + r) : 0;
    bf16* dst = p.out + r * p.H;
    const bool valid = s >= 0 && s < p.n && k >= 0 && k < p.P;
    if (s >= 0 && !valid && lane == 0) set_status(p.status, kStatusBadShape);
    const long srow = static_cast<long>(s) * p.P + k;
    for (long c = lane * 8; c < p.H; c += 256) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (valid) {
        if (!p.fp8) {
          v = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(p.payload) + srow * p.H + c);
        } else {
          const uint2 q = *reinterpret_cast<const uint2*>(p.payload + srow * p.H + c);
          float f[8];
          dequant8(q, p.pscale[srow * (p.H / 128) + c / 128], f);
          v = pack_bf16x8(f);
        }
      }
      *reinterpret_cast<uint4*>(dst + c) = v;
    }
  }
}

// ------------------------------------------------------------------ receiver: expert outputs -> e4m3 rows
struct EpQuantParams {
  const bf16* y;
  const int* rows_used;
  uint8_t* q;
  float* scale;
  long H, rows_cap;
  int stochastic;
  unsigned long long seed;
};

__global__ void __launch_bounds__(256) ep_quant_rows_kernel(const EpQuantParams p) {
  const int lane = threadIdx.x & 31;
  const long rows = min(static_cast<long>(*p.rows_used), p.rows_cap);
  const long nwarps = static_cast<long>(gridDim.x) * kWarps;
  for (long r = static_cast<long>(blockIdx.x) * kWarps + (threadIdx.x >> 5); r < rows; r += nwarps) {
    for (long c0 = 0; c0 < p.H; c0 += 256) {
      const long c = c0 + lane * 8;
      const bool act = c < p.H;
      float v[8];
      float amax = 0.f;
      if (act) {
        unpack_bf16x8(*reinterpret_cast<const uint4*>(p.y + r * p.H + c), v);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
      }
      amax = half_warp_max(amax);
      const float scale = amax > 0.f ? amax / 448.f : 1.f;
      if (act) {
        *reinterpret_cast<uint2*>(p.q + r * p.H + c) =
            quant8(v, scale, p.stochastic != 0, p.seed, static_cast<uint64_t>(r) * p.H + c);
        if ((lane & 15) == 0) p.scale[r * (p.H / 128) + c / 128] = scale;
      }
    }
  }
}

// ------------------------------------------------------------------ sender: pull + weighted sum over top-k
struct EpPullParams {
  int T, K, n;
  long H, P, rows_cap;
  const int* dest_tk;   // [T*K] destination rank of assignment (t, k)
  const int* slot_tk;   // [T*K] its row in the destination slab block
  const float* w_tk;    // [T*K] weight, nullptr = 1
  const int* pos_in;    // [T*K] grouped row at the destination (backward), nullptr = read the row map
  const int* rowmap[kEpMaxRanks];   // destination's row map, this source's block
  const uint8_t* src[kEpMaxRanks];  // destination's rows (bf16, or e4m3 when fp8)
  const float* src_scale[kEpMaxRanks];
  int fp8;
  bf16* out;      // [T, H]
  bf16* y_save;   // [T*K, H] pulled rows (zero when dropped), optional
  int* pos_out;   // [T*K] optional
  int* status;
};

__global__ void __launch_bounds__(256) ep_pull_kernel(const EpPullParams p) {
  const int lane = threadIdx.x & 31;
  const long nwarps = static_cast<long>(gridDim.x) * kWarps;
  for (long t = static_cast<long>(blockIdx.x) * kWarps + (threadIdx.x >> 5); t < p.T; t += nwarps) {
    int my_d = 0, my_pos = -1;
    float my_w = 0.f;
    if (lane < p.K) {
      const long a = t * p.K + lane;
      const int d = p.dest_tk[a];
      int pos = -1;
      if (d >= 0 && d < p.n) {
        if (p.pos_in) {
          pos = p.pos_in[a];
        } else {
          const int s = p.slot_tk[a];
          if (s >= 0 && s < p.P) pos = p.rowmap[d][s];
        }
        if (pos >= p.rows_cap) {
          set_status(p.status, kStatusBadShape);
          pos = -1;
        }
      } else {
        set_status(p.status, kStatusBadShape);
      }
      my_d = d;
      my_pos = pos < 0 ? -1 : pos;
      my_w = p.w_tk ? p.w_tk[a] : 1.f;
      if (p.pos_out) p.pos_out[a] = my_pos;
    }
    int dk[kEpMaxTopK], posk[kEpMaxTopK];
    float wk[kEpMaxTopK];
#pragma unroll
    for (int k = 0; k < kEpMaxTopK; ++k) {
      dk[k] = __shfl_sync(0xffffffffu, my_d, k);
      posk[k] = __shfl_sync(0xffffffffu, my_pos, k);
      wk[k] = __shfl_sync(0xffffffffu, my_w, k);
    }
    for (long c0 = 0; c0 < p.H; c0 += 256) {
      const long c = c0 + lane * 8;
      if (c >= p.H) continue;
      // All K rows are requested before any is used: K loads in flight per lane.
      uint4 raw[kEpMaxTopK];
#pragma unroll
      for (int k = 0; k < kEpMaxTopK; ++k) {
        raw[k] = make_uint4(0u, 0u, 0u, 0u);
        if (k < p.K && posk[k] >= 0) {
          const long row = posk[k];
          if (!p.fp8) {
            raw[k] = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(p.src[dk[k]]) + row * p.H + c);
          } else {
            const uint2 q = *reinterpret_cast<const uint2*>(p.src[dk[k]] + row * p.H + c);
            raw[k].x = q.x;
            raw[k].y = q.y;
            raw[k].z = __float_as_uint(p.src_scale[dk[k]][row * (p.H / 128) + c / 128]);
          }
        }
      }
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int k = 0; k < kEpMaxTopK; ++k) {
        if (k >= p.K) break;
        float v[8];
        if (p.fp8) {
          if (posk[k] >= 0) {
            dequant8(make_uint2(raw[k].x, raw[k].y), __uint_as_float(raw[k].z), v);
            raw[k] = pack_bf16x8(v);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = 0.f;
          }
        } else {
          unpack_bf16x8(raw[k], v);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = fmaf(wk[k], v[j], acc[j]);
        if (p.y_save) *reinterpret_cast<uint4*>(p.y_save + (t * p.K + k) * p.H + c) = raw[k];
      }
      *reinterpret_cast<uint4*>(p.out + t * p.H + c) = pack_bf16x8(acc);
    }
  }
}

// ------------------------------------------------------------------ receiver: combine backward
struct EpCombineBwdParams {
  const int* rows_used;
  const int* row_src;
  const int* row_tok;
  const float* row_w;
  const bf16* dout[kEpMaxRanks];  // every source's output gradient [T_src, H]
  bf16* dy;                       // [rows_cap, H]
  long H, rows_cap;
  int T, n;
  int* status;
};

__global__ void __launch_bounds__(256) ep_combine_bwd_kernel(const EpCombineBwdParams p) {
  const int lane = threadIdx.x & 31;
  const long rows = min(static_cast<long>(*p.rows_used), p.rows_cap);
  const long nwarps = static_cast<long>(gridDim.x) * kWarps;
  for (long r = static_cast<long>(blockIdx.x) * kWarps + (threadIdx.x >> 5); r < rows; r += nwarps) {
    const int s = __ldg(p.row_src + r);
    const int t = s >= 0 ? __ldg(p.row_tok + r) : 0;
    const bool valid = s >= 0 && s < p.n && t >= 0 && t < p.T;
    if (s >= 0 && !valid && lane == 0) set_status(p.status, kStatusBadShape);
    const float w = valid ? __ldg(p.row_w + r) : 0.f;
    const bf16* g = valid ? p.dout[s] + static_cast<long>(t) * p.H : nullptr;
    for (long c = lane * 8; c < p.H; c += 256) {
      float v[8];
      if (valid) {
        unpack_bf16x8(*reinterpret_cast<const uint4*>(g + c), v);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] *= w;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.f;
      }
      *reinterpret_cast<uint4*>(p.dy + r * p.H + c) = pack_bf16x8(v);
    }
  }
}

int row_grid(int dev, long rows) {
  const long want = (rows + kWarps - 1) / kWarps;
  const long cap = static_cast<long>(num_sms(dev)) * 8;
  return static_cast<int>(std::max<long>(1, std::min(want, cap)));
}

template <typename T>
void fill_ptrs(T* (&dst)[kEpMaxRanks], const std::vector<int64_t>& v, int64_t add_bytes = 0) {
  for (int i = 0; i < kEpMaxRanks; ++i)
    dst[i] = i < static_cast<int>(v.size()) && v[i] ? reinterpret_cast<T*>(v[i] + add_bytes) : nullptr;
}

void check_i32(const at::Tensor& t, int64_t n, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous() && t.numel() >= n, what,
              ": int32 contiguous CUDA tensor of at least ", n, " elements");
}

}  // namespace

// ------------------------------------------------------------------ host entry points
void ep_dispatch(const at::Tensor& x, const at::Tensor& idx, const at::Tensor& w, at::Tensor& dest_tk,
                 at::Tensor& slot_tk, const at::Tensor& ctr, int64_t epr, std::vector<int64_t> payload,
                 std::vector<int64_t> pscale, std::vector<int64_t> meta, std::vector<int64_t> flag,
                 std::vector<int64_t> info, const at::Tensor& done, int64_t P, int64_t epoch, bool fp8,
                 bool stochastic, int64_t seed) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
              "ep_dispatch: x bf16 [T, H] contiguous");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "ep_dispatch: x must be 16-byte aligned");
  const int n = static_cast<int>(payload.size());
  TORCH_CHECK(n >= 1 && n <= kEpMaxRanks && meta.size() == payload.size() && flag.size() == payload.size() &&
                  info.size() == payload.size(),
              "ep_dispatch: 1..8 destinations");
  const int64_t T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % (fp8 ? 128 : 8) == 0, "ep_dispatch: H must be a multiple of ", fp8 ? 128 : 8);
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kLong && idx.dim() == 2 && idx.size(0) == T &&
                  idx.is_contiguous(),
              "ep_dispatch: idx int64 [T, K]");
  const int64_t K = idx.size(1);
  TORCH_CHECK(T * K <= P && T * K < (1 << 20), "ep_dispatch: T * K must fit the slab block and 20 bits");
  TORCH_CHECK(w.is_cuda() && w.is_contiguous() && w.numel() == T * K &&
                  (w.scalar_type() == at::kFloat || w.scalar_type() == at::kBFloat16),
              "ep_dispatch: w [T, K] fp32 or bf16");
  check_i32(dest_tk, T * K, "ep_dispatch: dest_tk");
  check_i32(slot_tk, T * K, "ep_dispatch: slot_tk");
  check_i32(ctr, n, "ep_dispatch: ctr");
  TORCH_CHECK(done.is_cuda() && done.scalar_type() == at::kInt && done.numel() >= 1, "ep_dispatch: done int32");
  EpDispatchParams p{};
  p.x = reinterpret_cast<const bf16*>(x.data_ptr());
  p.H = H;
  p.T = static_cast<int>(T);
  p.K = static_cast<int>(K);
  p.epr = static_cast<int>(epr);
  p.idx = idx.data_ptr<int64_t>();
  p.w = w.data_ptr();
  p.w_f32 = w.scalar_type() == at::kFloat ? 1 : 0;
  p.dest_tk = dest_tk.data_ptr<int>();
  p.slot_tk = slot_tk.data_ptr<int>();
  p.ctr = ctr.data_ptr<int>();
  fill_ptrs(p.payload, payload);
  if (fp8) fill_ptrs(p.pscale, pscale);
  fill_ptrs(p.meta, meta);
  fill_ptrs(p.flag, flag);
  fill_ptrs(p.info, info);
  p.P = P;
  p.n = n;
  p.fp8 = fp8 ? 1 : 0;
  p.stochastic = stochastic ? 1 : 0;
  p.seed = static_cast<unsigned long long>(seed);
  p.done = reinterpret_cast<unsigned int*>(done.data_ptr());
  p.epoch = static_cast<unsigned long long>(epoch);
  const int dev = x.get_device();
  p.status = device_status(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  ep_dispatch_kernel<<<row_grid(dev, std::max<int64_t>(T * K, 1)), 256, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

void ep_recv_keys(int64_t meta_ptr, int64_t info_ptr, at::Tensor& keys, at::Tensor& counts, int64_t P, int64_t n,
                  int64_t epr, int64_t K) {
  TORCH_CHECK(keys.is_cuda() && keys.scalar_type() == at::kLong && keys.numel() == n * P, "ep_recv_keys: keys");
  check_i32(counts, epr, "ep_recv_keys: counts");
  TORCH_CHECK(epr >= 1 && epr <= 255 && n <= kEpMaxRanks && P < (1LL << 40), "ep_recv_keys: sizes");
  EpKeyParams p{};
  p.meta = reinterpret_cast<const int4*>(meta_ptr);
  p.info = reinterpret_cast<const int*>(info_ptr);
  p.keys = reinterpret_cast<long long*>(keys.data_ptr<int64_t>());
  p.counts = counts.data_ptr<int>();
  p.P = P;
  p.n = static_cast<int>(n);
  p.epr = static_cast<int>(epr);
  p.K = static_cast<int>(K);
  const int dev = keys.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  const long total = n * P;
  const int grid = static_cast<int>(std::max<long>(1, std::min<long>((total + 255) / 256, num_sms(dev) * 4)));
  ep_recv_keys_kernel<<<grid, 256, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

void ep_recv_layout(const at::Tensor& skeys, const at::Tensor& order, int64_t meta_ptr, int64_t info_ptr,
                    const at::Tensor& counts, at::Tensor& offsets, at::Tensor& row_src, at::Tensor& row_slot,
                    at::Tensor& row_tok, at::Tensor& row_w, int64_t rowmap_ptr, at::Tensor& stats, int64_t P,
                    int64_t n, int64_t epr, int64_t K, int64_t E, double capacity_factor, int64_t host_cap) {
  const int64_t rows = row_src.numel();
  TORCH_CHECK(skeys.scalar_type() == at::kLong && order.scalar_type() == at::kLong && skeys.numel() == n * P &&
                  order.numel() == n * P,
              "ep_recv_layout: sorted keys / order int64 [n * P]");
  check_i32(counts, epr, "ep_recv_layout: counts");
  check_i32(offsets, epr + 1, "ep_recv_layout: offsets");
  check_i32(row_slot, rows, "ep_recv_layout: row_slot");
  check_i32(row_tok, rows, "ep_recv_layout: row_tok");
  TORCH_CHECK(row_w.scalar_type() == at::kFloat && row_w.numel() == rows && stats.scalar_type() == at::kFloat &&
                  stats.numel() == 2,
              "ep_recv_layout: row_w / stats fp32");
  TORCH_CHECK(epr >= 1 && epr <= 255, "ep_recv_layout: at most 255 local experts");
  EpLayoutParams p{};
  p.skeys = reinterpret_cast<const long long*>(skeys.data_ptr<int64_t>());
  p.order = order.data_ptr<int64_t>();
  p.meta = reinterpret_cast<const int4*>(meta_ptr);
  p.info = reinterpret_cast<const int*>(info_ptr);
  p.counts = counts.data_ptr<int>();
  p.offsets = offsets.data_ptr<int>();
  p.row_src = row_src.data_ptr<int>();
  p.row_slot = row_slot.data_ptr<int>();
  p.row_tok = row_tok.data_ptr<int>();
  p.row_w = row_w.data_ptr<float>();
  p.rowmap = reinterpret_cast<int*>(rowmap_ptr);
  p.stats = stats.data_ptr<float>();
  p.P = P;
  p.rows = rows;
  p.n = static_cast<int>(n);
  p.epr = static_cast<int>(epr);
  p.K = static_cast<int>(K);
  p.E = static_cast<int>(E);
  p.capacity_factor = capacity_factor;
  p.host_cap = host_cap;
  const int dev = skeys.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  const long work = std::max<long>(n * P, rows);
  const int grid = static_cast<int>(std::max<long>(1, std::min<long>((work + 255) / 256, num_sms(dev) * 4)));
  ep_recv_layout_kernel<<<grid, 256, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

void ep_wait(int64_t flags_ptr, int64_t n, int64_t epoch, int64_t device) {
  TORCH_CHECK(n >= 1 && n <= kEpMaxRanks, "ep_wait: 1..8 flags");
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(static_cast<int>(device));
  ep_wait_kernel<<<1, 32, 0, stream>>>(reinterpret_cast<const unsigned long long*>(flags_ptr), static_cast<int>(n),
                                       static_cast<unsigned long long>(epoch), device_status(static_cast<int>(device)));
  NTB_LAUNCH_CHECK(1);
}

void ep_signal(std::vector<int64_t> flag, int64_t epoch, int64_t device) {
  TORCH_CHECK(flag.size() >= 1 && flag.size() <= kEpMaxRanks, "ep_signal: 1..8 flags");
  EpSignalParams p{};
  fill_ptrs(p.flag, flag);
  p.n = static_cast<int>(flag.size());
  p.epoch = static_cast<unsigned long long>(epoch);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(static_cast<int>(device));
  ep_signal_kernel<<<1, 32, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

void ep_gather(at::Tensor& out, const at::Tensor& rows_used, const at::Tensor& row_src, const at::Tensor& row_slot,
               int64_t payload_ptr, int64_t scale_ptr, int64_t P, int64_t n, bool fp8) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.is_contiguous(),
              "ep_gather: out bf16 [R, H]");
  const int64_t R = out.size(0), H = out.size(1);
  TORCH_CHECK(H % (fp8 ? 128 : 8) == 0, "ep_gather: H alignment");
  check_i32(row_src, R, "ep_gather: row_src");
  check_i32(row_slot, R, "ep_gather: row_slot");
  check_i32(rows_used, 1, "ep_gather: rows_used");
  EpGatherParams p{};
  p.payload = reinterpret_cast<const uint8_t*>(payload_ptr);
  p.pscale = reinterpret_cast<const float*>(scale_ptr);
  p.rows_used = rows_used.data_ptr<int>();
  p.row_src = row_src.data_ptr<int>();
  p.row_slot = row_slot.data_ptr<int>();
  p.out = reinterpret_cast<bf16*>(out.data_ptr());
  p.H = H;
  p.P = P;
  p.rows_cap = R;
  p.n = static_cast<int>(n);
  p.fp8 = fp8 ? 1 : 0;
  const int dev = out.get_device();
  p.status = device_status(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  ep_gather_kernel<<<row_grid(dev, std::max<int64_t>(R, 1)), 256, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

void ep_quant_rows(const at::Tensor& y, const at::Tensor& rows_used, int64_t q_ptr, int64_t scale_ptr,
                   bool stochastic, int64_t seed) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.dim() == 2 && y.is_contiguous() &&
                  y.size(1) % 128 == 0,
              "ep_quant_rows: y bf16 [R, H], H % 128 == 0");
  check_i32(rows_used, 1, "ep_quant_rows: rows_used");
  EpQuantParams p{};
  p.y = reinterpret_cast<const bf16*>(y.data_ptr());
  p.rows_used = rows_used.data_ptr<int>();
  p.q = reinterpret_cast<uint8_t*>(q_ptr);
  p.scale = reinterpret_cast<float*>(scale_ptr);
  p.H = y.size(1);
  p.rows_cap = y.size(0);
  p.stochastic = stochastic ? 1 : 0;
  p.seed = static_cast<unsigned long long>(seed);
  const int dev = y.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  ep_quant_rows_kernel<<<row_grid(dev, std::max<int64_t>(y.size(0), 1)), 256, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

void ep_pull(at::Tensor& out, const at::Tensor& dest_tk, const at::Tensor& slot_tk,
             const c10::optional<at::Tensor>& w_tk, const c10::optional<at::Tensor>& pos_in,
             std::vector<int64_t> rowmap, std::vector<int64_t> src, std::vector<int64_t> src_scale, int64_t P,
             int64_t rows_cap, bool fp8, const c10::optional<at::Tensor>& y_save,
             const c10::optional<at::Tensor>& pos_out) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.is_contiguous(),
              "ep_pull: out bf16 [T, H]");
  const int64_t T = out.size(0), H = out.size(1);
  const int n = static_cast<int>(src.size());
  TORCH_CHECK(n >= 1 && n <= kEpMaxRanks, "ep_pull: 1..8 sources");
  TORCH_CHECK(H % (fp8 ? 128 : 8) == 0, "ep_pull: H alignment");
  TORCH_CHECK(T > 0 && dest_tk.numel() % T == 0, "ep_pull: dest_tk must hold T * K entries");
  const int64_t K = dest_tk.numel() / T;
  TORCH_CHECK(K >= 1 && K <= kEpMaxTopK, "ep_pull: top-k in [1, 8]");
  check_i32(dest_tk, T * K, "ep_pull: dest_tk");
  EpPullParams p{};
  p.T = static_cast<int>(T);
  p.K = static_cast<int>(K);
  p.n = n;
  p.H = H;
  p.P = P;
  p.rows_cap = rows_cap;
  p.dest_tk = dest_tk.data_ptr<int>();
  if (pos_in.has_value()) {
    check_i32(*pos_in, T * K, "ep_pull: pos_in");
    p.pos_in = pos_in->data_ptr<int>();
  } else {
    check_i32(slot_tk, T * K, "ep_pull: slot_tk");
    p.slot_tk = slot_tk.data_ptr<int>();
    TORCH_CHECK(static_cast<int>(rowmap.size()) == n, "ep_pull: one row map per source");
    fill_ptrs(p.rowmap, rowmap);
  }
  if (w_tk.has_value()) {
    TORCH_CHECK(w_tk->is_cuda() && w_tk->scalar_type() == at::kFloat && w_tk->is_contiguous() &&
                    w_tk->numel() >= T * K,
                "ep_pull: w fp32 [T * K]");
    p.w_tk = w_tk->data_ptr<float>();
  }
  fill_ptrs(p.src, src);
  if (fp8) fill_ptrs(p.src_scale, src_scale);
  p.fp8 = fp8 ? 1 : 0;
  p.out = reinterpret_cast<bf16*>(out.data_ptr());
  if (y_save.has_value()) {
    TORCH_CHECK(y_save->scalar_type() == at::kBFloat16 && y_save->is_contiguous() && y_save->numel() >= T * K * H,
                "ep_pull: y_save bf16 [T * K, H]");
    p.y_save = reinterpret_cast<bf16*>(y_save->data_ptr());
  }
  if (pos_out.has_value()) {
    check_i32(*pos_out, T * K, "ep_pull: pos_out");
    p.pos_out = pos_out->data_ptr<int>();
  }
  const int dev = out.get_device();
  p.status = device_status(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  ep_pull_kernel<<<row_grid(dev, T), 256, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

void ep_combine_bwd(at::Tensor& dy, const at::Tensor& rows_used, const at::Tensor& row_src, const at::Tensor& row_tok,
                    const at::Tensor& row_w, std::vector<int64_t> dout, int64_t T) {
  TORCH_CHECK(dy.is_cuda() && dy.scalar_type() == at::kBFloat16 && dy.dim() == 2 && dy.is_contiguous() &&
                  dy.size(1) % 8 == 0,
              "ep_combine_bwd: dy bf16 [R, H]");
  const int64_t R = dy.size(0);
  const int n = static_cast<int>(dout.size());
  TORCH_CHECK(n >= 1 && n <= kEpMaxRanks, "ep_combine_bwd: 1..8 sources");
  check_i32(rows_used, 1, "ep_combine_bwd: rows_used");
  check_i32(row_src, R, "ep_combine_bwd: row_src");
  check_i32(row_tok, R, "ep_combine_bwd: row_tok");
  TORCH_CHECK(row_w.is_cuda() && row_w.scalar_type() == at::kFloat && row_w.numel() >= R, "ep_combine_bwd: row_w");
  EpCombineBwdParams p{};
  p.rows_used = rows_used.data_ptr<int>();
  p.row_src = row_src.data_ptr<int>();
  p.row_tok = row_tok.data_ptr<int>();
  p.row_w = row_w.data_ptr<float>();
  fill_ptrs(p.dout, dout);
  p.dy = reinterpret_cast<bf16*>(dy.data_ptr());
  p.H = dy.size(1);
  p.rows_cap = R;
  p.T = static_cast<int>(T);
  p.n = n;
  const int dev = dy.get_device();
  p.status = device_status(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  ep_combine_bwd_kernel<<<row_grid(dev, std::max<int64_t>(R, 1)), 256, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

}  // namespace ntb
