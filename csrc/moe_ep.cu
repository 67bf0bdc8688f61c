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
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float y = fminf(fmaxf(v[j] / s, -448.f), 448.f);
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
  const bf16* x;  // [T, H] this rank's tokens
  long H;
  int T;
  int n_assign;             // T * K
  const int* tok;           // token of each destination-sorted assignment
  const int* dest;          // destination rank
  const int* slot;          // row inside this source's block of the destination slab
  const int* lexp;          // expert index local to the destination
  const int* kslot;         // top-k slot of the assignment
  const float* w;           // routing weight (fp32)
  const int* send_counts;   // [n] rows sent to each destination
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

__global__ void __launch_bounds__(256) ep_dispatch_kernel(const EpDispatchParams p) {
  const int lane = threadIdx.x & 31;
  const long nwarps = static_cast<long>(gridDim.x) * kWarps;
  for (long i = static_cast<long>(blockIdx.x) * kWarps + (threadIdx.x >> 5); i < p.n_assign; i += nwarps) {
    const int t = __ldg(p.tok + i), d = __ldg(p.dest + i), s = __ldg(p.slot + i);
    if (t < 0 || t >= p.T || d < 0 || d >= p.n || s < 0 || s >= p.P) {
      if (lane == 0) set_status(p.status, kStatusBadShape);
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
              quant8(v, scale, p.stochastic != 0, p.seed, static_cast<uint64_t>(i) * p.H + c);
          if ((lane & 15) == 0) sc[c / 128] = scale;
        }
      }
    }
    if (lane == 0)
      p.meta[d][s] = make_int4(__ldg(p.lexp + i), t, __float_as_int(__ldg(p.w + i)), __ldg(p.kslot + i));
  }
  // The last CTA to finish publishes: counts, then the epoch, to every destination.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < p.n; ++d) {
        p.info[d][0] = p.send_counts[d];
        p.info[d][1] = p.T;
      }
      __threadfence_system();
      for (int d = 0; d < p.n; ++d) st_release_sys_u64(p.flag[d], p.epoch);
      *p.done = 0u;
    }
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
  for (int d = 0; d < p.n; ++d) st_release_sys_u64(p.flag[d], p.epoch);
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
void ep_dispatch(const at::Tensor& x, const at::Tensor& tok, const at::Tensor& dest, const at::Tensor& slot,
                 const at::Tensor& lexp, const at::Tensor& kslot, const at::Tensor& w, const at::Tensor& send_counts,
                 std::vector<int64_t> payload, std::vector<int64_t> pscale, std::vector<int64_t> meta,
                 std::vector<int64_t> flag, std::vector<int64_t> info, const at::Tensor& done, int64_t P,
                 int64_t epoch, bool fp8, bool stochastic, int64_t seed) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
              "ep_dispatch: x bf16 [T, H] contiguous");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "ep_dispatch: x must be 16-byte aligned");
  const int n = static_cast<int>(payload.size());
  TORCH_CHECK(n >= 1 && n <= kEpMaxRanks && meta.size() == payload.size() && flag.size() == payload.size() &&
                  info.size() == payload.size(),
              "ep_dispatch: 1..8 destinations");
  const int64_t H = x.size(1), nA = tok.numel();
  TORCH_CHECK(H % (fp8 ? 128 : 8) == 0, "ep_dispatch: H must be a multiple of ", fp8 ? 128 : 8);
  for (const at::Tensor* t : {&tok, &dest, &slot, &lexp, &kslot}) check_i32(*t, nA, "ep_dispatch");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kFloat && w.numel() >= nA, "ep_dispatch: w fp32");
  check_i32(send_counts, n, "ep_dispatch: send_counts");
  TORCH_CHECK(done.is_cuda() && done.scalar_type() == at::kInt && done.numel() >= 1, "ep_dispatch: done int32");
  EpDispatchParams p{};
  p.x = reinterpret_cast<const bf16*>(x.data_ptr());
  p.H = H;
  p.T = static_cast<int>(x.size(0));
  p.n_assign = static_cast<int>(nA);
  p.tok = tok.data_ptr<int>();
  p.dest = dest.data_ptr<int>();
  p.slot = slot.data_ptr<int>();
  p.lexp = lexp.data_ptr<int>();
  p.kslot = kslot.data_ptr<int>();
  p.w = w.data_ptr<float>();
  p.send_counts = send_counts.data_ptr<int>();
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
  ep_dispatch_kernel<<<row_grid(dev, std::max<int64_t>(nA, 1)), 256, 0, stream>>>(p);
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
