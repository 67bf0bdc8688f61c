// Fused ZeRO-1/2 optimizer step for data parallelism inside one NVLink node.
//
// Every rank keeps its flat parameter (bf16) and gradient (fp32) buffers in
// symmetric memory (CUDA IPC); rank r owns the shard [r * chunk, (r+1) * chunk)
// of every buffer. A step is three launches per rank, no NCCL:
//
//   zero_rs_kernel    after every rank's "gradients ready" flag: this rank's
//                     shard of every buffer is summed over the ranks by reading
//                     the peers' gradient buffers over NVLink (the reduce-
//                     scatter), written in place into the local gradient shard,
//                     with the sum of squares for gradient clipping. The last
//                     CTA pushes the partial sum of squares into every peer's
//                     slot and publishes it (system-scope release).
//   zero_adam_kernel  waits for every rank's partial, forms the clip
//                     coefficient x 1/dp on the device, applies AdamW to the
//                     fp32 master shard and moments, and stores the new bf16
//                     shard into EVERY rank's parameter buffer (peer stores:
//                     the all-gather); the last CTA publishes "parameters
//                     written".
//   a bounded wait    for every rank's "parameters written" before the next
//                     use of the parameters.
//
// Ordering: a rank reads a peer's gradients only after that peer's "gradients
// ready" (its backward finished); a rank starts its update only after every
// peer published its partial norm, i.e. finished reading this rank's
// gradients, so zeroing the gradients afterwards is safe; a peer writes this
// rank's parameters only after this rank's backward finished. Every wait is
// bounded and reports through the status word.
//
// AdamW (decoupled weight decay, bias-corrected), the same update as the flat
// optimizer's kernel: p *= 1 - lr wd; m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2;
// p -= (lr / bc1) m / (sqrt(v) / sqrt(bc2) + eps), g = grad x scale.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"
#include "peer.cuh"

#include <cmath>
#include <vector>

namespace ntb {
namespace {

using bf16 = __nv_bfloat16;
constexpr int kZMaxRanks = 8;
constexpr int kZMaxBufs = 32;

struct ZeroBuf {
  const float* grad[kZMaxRanks];  // rank r's gradient buffer at this rank's shard offset
  bf16* param[kZMaxRanks];        // rank r's parameter buffer at this rank's shard offset
  float* red;                     // this rank's gradient shard (reduced in place)
  float* master;
  float* m;
  float* v;
  long n;                         // shard elements (multiple of 8)
  float lr, wd;
  int cls;                        // 0: norm class summed over every group, 1: replicated class
};

struct ZeroParams {
  ZeroBuf b[kZMaxBufs];
  int nbuf, n, me;
  float* stats_acc;                            // local [2] accumulator (zero at rest)
  float* stats_slot[kZMaxRanks];               // rank r's slot for this rank's partial [2]
  const float* stats_in;                       // local [8][2] partials of every rank
  unsigned long long* flag_stats[kZMaxRanks];  // rank r's STATS flag for this rank
  unsigned long long* flag_params[kZMaxRanks]; // rank r's PARAMS flag for this rank
  const unsigned long long* my_stats_flags;    // local STATS flags [8]
  unsigned int* done;                          // local arrival counter (zero at rest)
  unsigned long long epoch;
  int publish;  // reduce-scatter: 1 = the last CTA publishes the partial sums (the step's last bucket)
  // update
  float b1, b2, eps, bc1, sqrt_bc2, inv_dp, max_norm;
  float* grad_norm;  // out [1]
  float* scale_out;  // out [1]
  int* status;
};

__device__ __forceinline__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) sh[w] = v;
  __syncthreads();
  float r = 0.f;
  if (threadIdx.x == 0)
    for (int i = 0; i < (blockDim.x >> 5); ++i) r += sh[i];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(256) zero_rs_kernel(const __grid_constant__ ZeroParams p) {
  __shared__ float sh[32];
  float ss[2] = {0.f, 0.f};
  for (int bi = 0; bi < p.nbuf; ++bi) {
    const ZeroBuf& b = p.b[bi];
    const long n4 = b.n / 4;
    float acc_ss = 0.f;
    for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
      float4 v[kZMaxRanks];
#pragma unroll
      for (int r = 0; r < kZMaxRanks; ++r)
        if (r < p.n) v[r] = reinterpret_cast<const float4*>(b.grad[r])[i];
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < kZMaxRanks; ++r)
        if (r < p.n) {  // fixed rank order: every rank sums its shard the same way
          s.x += v[r].x;
          s.y += v[r].y;
          s.z += v[r].z;
          s.w += v[r].w;
        }
      reinterpret_cast<float4*>(b.red)[i] = s;
      acc_ss += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
    }
    ss[b.cls] += acc_ss;
  }
  const float s0 = block_sum(ss[0], sh);
  const float s1 = block_sum(ss[1], sh);
  if (threadIdx.x == 0) {
    atomicAdd(p.stats_acc, s0);
    atomicAdd(p.stats_acc + 1, s1);
    __threadfence_system();
    const unsigned int prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x - 1 && !p.publish) {
      *p.done = 0u;  // an earlier bucket of the step: the sums stay in stats_acc for the next launch
    } else if (prev == gridDim.x - 1) {
      __threadfence_system();
      const float a0 = atomicAdd(p.stats_acc, 0.f), a1 = atomicAdd(p.stats_acc + 1, 0.f);
      for (int r = 0; r < p.n; ++r) {
        p.stats_slot[r][0] = a0;
        p.stats_slot[r][1] = a1;
      }
      __threadfence_system();
      for (int r = 0; r < p.n; ++r) st_relaxed_sys_u64(p.flag_stats[r], p.epoch);
      p.stats_acc[0] = 0.f;
      p.stats_acc[1] = 0.f;
      *p.done = 0u;
    }
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(256) zero_adam_kernel(const __grid_constant__ ZeroParams p) {
  __shared__ float s_scale;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int r = 0; r < p.n && ok; ++r)
      ok = spin_until([&] { return ld_acquire_sys_u64(p.my_stats_flags + r) >= p.epoch; }, p.status,
                      kStatusTimeoutPeer);
    float total = 0.f;
    if (ok)
      for (int r = 0; r < p.n; ++r) {
        const float* st = p.stats_in + 2 * r;
        total += *reinterpret_cast<const volatile float*>(st) + *reinterpret_cast<const volatile float*>(st + 1);
      }
    const float norm = sqrtf(total) * p.inv_dp;
    float coef = 1.f;
    if (p.max_norm > 0.f) coef = fminf(p.max_norm / (norm + 1e-6f), 1.f);
    s_scale = coef * p.inv_dp;
    s_ok = ok ? 1 : 0;
    if (blockIdx.x == 0 && ok) {
      if (p.grad_norm) *p.grad_norm = norm;
      if (p.scale_out) *p.scale_out = s_scale;
    }
  }
  __syncthreads();
  if (s_ok) {
    const float gs = s_scale;
    for (int bi = 0; bi < p.nbuf; ++bi) {
      const ZeroBuf& b = p.b[bi];
      const float step = b.lr / p.bc1, decay = 1.f - b.lr * b.wd;
      const long n8 = b.n / 8;
      for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
           i += static_cast<long>(gridDim.x) * blockDim.x) {
        float P[8], M[8], V[8], G[8];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float4 pp = reinterpret_cast<const float4*>(b.master)[2 * i + h];
          const float4 mm = reinterpret_cast<const float4*>(b.m)[2 * i + h];
          const float4 vv = reinterpret_cast<const float4*>(b.v)[2 * i + h];
          const float4 gg = reinterpret_cast<const float4*>(b.red)[2 * i + h];
          P[4 * h] = pp.x; P[4 * h + 1] = pp.y; P[4 * h + 2] = pp.z; P[4 * h + 3] = pp.w;
          M[4 * h] = mm.x; M[4 * h + 1] = mm.y; M[4 * h + 2] = mm.z; M[4 * h + 3] = mm.w;
          V[4 * h] = vv.x; V[4 * h + 1] = vv.y; V[4 * h + 2] = vv.z; V[4 * h + 3] = vv.w;
          G[4 * h] = gg.x; G[4 * h + 1] = gg.y; G[4 * h + 2] = gg.z; G[4 * h + 3] = gg.w;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float g = G[j] * gs;
          P[j] *= decay;
          M[j] = p.b1 * M[j] + (1.f - p.b1) * g;
          V[j] = p.b2 * V[j] + (1.f - p.b2) * g * g;
          P[j] -= step * M[j] / (sqrtf(V[j]) / p.sqrt_bc2 + p.eps);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          reinterpret_cast<float4*>(b.master)[2 * i + h] =
              make_float4(P[4 * h], P[4 * h + 1], P[4 * h + 2], P[4 * h + 3]);
          reinterpret_cast<float4*>(b.m)[2 * i + h] = make_float4(M[4 * h], M[4 * h + 1], M[4 * h + 2], M[4 * h + 3]);
          reinterpret_cast<float4*>(b.v)[2 * i + h] = make_float4(V[4 * h], V[4 * h + 1], V[4 * h + 2], V[4 * h + 3]);
        }
        const uint4 o = make_uint4(pack2(P[0], P[1]), pack2(P[2], P[3]), pack2(P[4], P[5]), pack2(P[6], P[7]));
#pragma unroll
        for (int r = 0; r < kZMaxRanks; ++r)
          if (r < p.n) reinterpret_cast<uint4*>(b.param[r])[i] = o;  // local and peer stores: the all-gather
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int r = 0; r < p.n; ++r) st_relaxed_sys_u64(p.flag_params[r], p.epoch);
      *p.done = 0u;
    }
  }
}

template <typename T>
void fill8(T* (&dst)[kZMaxRanks], const std::vector<int64_t>& v) {
  for (int i = 0; i < kZMaxRanks; ++i) dst[i] = i < static_cast<int>(v.size()) ? reinterpret_cast<T*>(v[i]) : nullptr;
}

ZeroParams make_params(const std::vector<std::vector<int64_t>>& grad_ptrs,
                       const std::vector<std::vector<int64_t>>& param_ptrs, const std::vector<at::Tensor>& red,
                       const std::vector<at::Tensor>& master, const std::vector<at::Tensor>& m,
                       const std::vector<at::Tensor>& v, const std::vector<double>& lr, const std::vector<double>& wd,
                       const std::vector<int64_t>& cls, int64_t me) {
  const int nb = static_cast<int>(red.size());
  TORCH_CHECK(nb >= 1 && nb <= kZMaxBufs, "zero_fused: 1..8 buffers");
  TORCH_CHECK(grad_ptrs.size() == red.size() && param_ptrs.size() == red.size() && master.size() == red.size() &&
                  m.size() == red.size() && v.size() == red.size() && lr.size() == red.size() &&
                  wd.size() == red.size() && cls.size() == red.size(),
              "zero_fused: per-buffer lists must have the same length");
  ZeroParams p{};
  p.nbuf = nb;
  p.n = static_cast<int>(grad_ptrs[0].size());
  TORCH_CHECK(p.n >= 1 && p.n <= kZMaxRanks && me >= 0 && me < p.n, "zero_fused: 1..8 ranks");
  p.me = static_cast<int>(me);
  for (int i = 0; i < nb; ++i) {
    const int64_t n = red[i].numel();
    TORCH_CHECK(n % 8 == 0, "zero_fused: shard sizes must be multiples of 8");
    for (const at::Tensor* t : {&red[i], &master[i], &m[i], &v[i]})
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == n &&
                      (reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0,
                  "zero_fused: fp32 contiguous 16-byte aligned shard tensors of equal size");
    TORCH_CHECK(static_cast<int>(grad_ptrs[i].size()) == p.n && static_cast<int>(param_ptrs[i].size()) == p.n,
                "zero_fused: one pointer per rank");
    for (int r = 0; r < p.n; ++r)
      TORCH_CHECK((grad_ptrs[i][r] & 15) == 0 && (param_ptrs[i][r] & 15) == 0, "zero_fused: 16-byte aligned peers");
    ZeroBuf& b = p.b[i];
    fill8(b.grad, grad_ptrs[i]);
    fill8(b.param, param_ptrs[i]);
    b.red = red[i].data_ptr<float>();
    b.master = master[i].data_ptr<float>();
    b.m = m[i].data_ptr<float>();
    b.v = v[i].data_ptr<float>();
    b.n = n;
    b.lr = static_cast<float>(lr[i]);
    b.wd = static_cast<float>(wd[i]);
    b.cls = cls[i] ? 1 : 0;
  }
  return p;
}

int zero_grid(int dev) { return num_sms(dev) * 4; }

}  // namespace

// Reduce-scatter (pull) of this rank's gradient shards + the clipping partials.
// publish = false: an earlier bucket of a step whose buffers are reduced one launch per bucket
// (while the backward still runs); its sums of squares stay in stats_acc for the last launch.
// grid = 0: the default (4 CTAs per SM); a bucket reduced under the backward uses a few CTAs.
void zero_reduce_scatter(std::vector<std::vector<int64_t>> grad_ptrs, const std::vector<at::Tensor>& red,
                         std::vector<int64_t> cls, at::Tensor& stats_acc, std::vector<int64_t> stats_slots,
                         std::vector<int64_t> flag_stats, const at::Tensor& done, int64_t me, int64_t epoch,
                         bool publish, int64_t grid) {
  TORCH_CHECK(!grad_ptrs.empty(), "zero_reduce_scatter: no buffers");
  std::vector<std::vector<int64_t>> param_ptrs(grad_ptrs.size(), std::vector<int64_t>(grad_ptrs[0].size(), 0));
  std::vector<double> z(red.size(), 0.0);
  ZeroParams p = make_params(grad_ptrs, param_ptrs, red, red, red, red, z, z, cls, me);
  TORCH_CHECK(stats_acc.scalar_type() == at::kFloat && stats_acc.numel() >= 2, "zero_reduce_scatter: stats_acc");
  p.stats_acc = stats_acc.data_ptr<float>();
  fill8(p.stats_slot, stats_slots);
  fill8(p.flag_stats, flag_stats);
  p.done = reinterpret_cast<unsigned int*>(done.data_ptr());
  p.epoch = static_cast<unsigned long long>(epoch);
  p.publish = publish ? 1 : 0;
  const int dev = red[0].get_device();
  p.status = device_status(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  zero_rs_kernel<<<grid > 0 ? static_cast<int>(grid) : zero_grid(dev), 256, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

// AdamW on this rank's shards + the parameter all-gather by peer stores.
void zero_adam_allgather(std::vector<std::vector<int64_t>> param_ptrs, const std::vector<at::Tensor>& red,
                         const std::vector<at::Tensor>& master, const std::vector<at::Tensor>& m,
                         const std::vector<at::Tensor>& v, std::vector<double> lr, std::vector<double> wd,
                         int64_t stats_in_ptr, int64_t my_stats_flags_ptr, std::vector<int64_t> flag_params,
                         const at::Tensor& done, int64_t me, int64_t epoch, double b1, double b2, double eps,
                         int64_t step, double inv_dp, double max_norm, at::Tensor& grad_norm, at::Tensor& scale_out) {
  TORCH_CHECK(!param_ptrs.empty(), "zero_adam_allgather: no buffers");
  std::vector<std::vector<int64_t>> grad_ptrs(param_ptrs.size(), std::vector<int64_t>(param_ptrs[0].size(), 0));
  std::vector<int64_t> cls(red.size(), 0);
  ZeroParams p = make_params(grad_ptrs, param_ptrs, red, master, m, v, lr, wd, cls, me);
  p.stats_in = reinterpret_cast<const float*>(stats_in_ptr);
  p.my_stats_flags = reinterpret_cast<const unsigned long long*>(my_stats_flags_ptr);
  fill8(p.flag_params, flag_params);
  p.done = reinterpret_cast<unsigned int*>(done.data_ptr());
  p.epoch = static_cast<unsigned long long>(epoch);
  p.b1 = static_cast<float>(b1);
  p.b2 = static_cast<float>(b2);
  p.eps = static_cast<float>(eps);
  p.bc1 = static_cast<float>(1.0 - std::pow(b1, static_cast<double>(step)));
  p.sqrt_bc2 = static_cast<float>(std::sqrt(1.0 - std::pow(b2, static_cast<double>(step))));
  p.inv_dp = static_cast<float>(inv_dp);
  p.max_norm = static_cast<float>(max_norm);
  TORCH_CHECK(grad_norm.scalar_type() == at::kFloat && scale_out.scalar_type() == at::kFloat, "zero_adam: fp32 outs");
  p.grad_norm = grad_norm.data_ptr<float>();
  p.scale_out = scale_out.data_ptr<float>();
  const int dev = red[0].get_device();
  p.status = device_status(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  zero_adam_kernel<<<zero_grid(dev), 256, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

}  // namespace ntb
