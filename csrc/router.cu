// Fused DeepSeek top-k router for sm_100a: one warp per token.
//
// Forward, from the router logits [T, E]:
//   scores  s = sigmoid(x) or softmax(x) (fp32 math, rounded to the logits
//           dtype like the unfused module's .to(dtype));
//   group-limited routing: group score = max inside the group, keep the
//           top `topk_group` groups, other experts are out of the running;
//   top-k   K rounds of a warp arg-max (ties -> lower expert index);
//   weights sigmoid: v / sum(v) when norm_topk_prob, softmax: softmax(v),
//           times routed_scaling_factor (bf16 rounding between the steps as
//           the unfused module performs them);
//   stats   counts[e] += #tokens choosing e, psum[e] += normalised score
//           (s / sum(s) for sigmoid, s for softmax): the aux loss is
//           E * sum_e counts_e / (T K) * psum_e / T.
// Backward: dlogits from dW [T, K] and dPsum [E] (the aux-loss gradient per
//   expert), through the weight normalisation, the score scatter and the
//   sigmoid / softmax Jacobian, in fp32.
//
// Reference parity: src/models/moe.py:196-350 (TopKRouter), the same
// selection rule and normalisations.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace ntb {
namespace {

using bf16 = __nv_bfloat16;
constexpr int kMaxE = 512;  // experts per router (16 per lane)
constexpr int kPer = kMaxE / 32;
constexpr int kMaxK = 8;
constexpr int kMaxGroups = 32;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<bf16>(bf16 v) { return __bfloat162float(v); }

// Rounds an fp32 value to the storage dtype and back (identity for fp32).
template <typename T>
__device__ __forceinline__ float rnd(float v);
template <>
__device__ __forceinline__ float rnd<float>(float v) { return v; }
template <>
__device__ __forceinline__ float rnd<bf16>(float v) { return __bfloat162float(__float2bfloat16(v)); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16(v); }

struct RouterCfg {
  int T, E, K;
  int softmax;        // 1: softmax scoring, 0: sigmoid
  int n_group, topk_group;
  int norm_topk;      // sigmoid only
  float scale;        // routed_scaling_factor
};

// Expert e of lane l: e = j * 32 + lane (j < kPer).
__device__ __forceinline__ void warp_argmax(float v, int e, float& bv, int& be) {
  bv = v;
  be = e;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oe = __shfl_xor_sync(0xffffffffu, be, o);
    if (ov > bv || (ov == bv && oe < be)) {
      bv = ov;
      be = oe;
    }
  }
}

// Computes the rounded scores of one token into s[] (lane-strided) and returns through
// `sel` / `selv` the K chosen experts and their score values.
template <typename T>
__device__ __forceinline__ void route_token(const T* __restrict__ x, const RouterCfg& c, int lane, float (&s)[kPer],
                                            int (&sel)[kMaxK], float (&selv)[kMaxK]) {
  const float NEG = -INFINITY;
  float xv[kPer];
  float mx = NEG;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = j * 32 + lane;
    xv[j] = e < c.E ? to_f(x[e]) : NEG;
    mx = fmaxf(mx, xv[j]);
  }
  if (c.softmax) {
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = j * 32 + lane;
      s[j] = e < c.E ? expf(xv[j] - mx) : 0.f;
      sum += s[j];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int j = 0; j < kPer; ++j) s[j] = rnd<T>(s[j] * inv);
  } else {
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = j * 32 + lane;
      s[j] = e < c.E ? rnd<T>(1.f / (1.f + expf(-xv[j]))) : 0.f;
    }
  }
  // Group-limited routing: eligible[j] marks experts of kept groups.
  bool elig[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) elig[j] = (j * 32 + lane) < c.E;
  if (c.n_group > 1 && c.topk_group < c.n_group) {
    const int epg = c.E / c.n_group;
    float gmax[kMaxGroups];
    for (int g = 0; g < c.n_group; ++g) gmax[g] = NEG;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = j * 32 + lane;
      if (e < c.E) gmax[e / epg] = fmaxf(gmax[e / epg], s[j]);
    }
    for (int g = 0; g < c.n_group; ++g) gmax[g] = warp_max(gmax[g]);
    uint32_t keep = 0u;
    for (int r = 0; r < c.topk_group; ++r) {
      int bg = -1;
      float bv = NEG;
      for (int g = 0; g < c.n_group; ++g)
        if (!(keep >> g & 1u) && (bg < 0 || gmax[g] > bv)) {
          bv = gmax[g];
          bg = g;
        }
      keep |= 1u << bg;
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = j * 32 + lane;
      if (e < c.E) elig[j] = keep >> (e / epg) & 1u;
    }
  }
  // Top-k: K rounds of a warp arg-max over the eligible, not yet chosen experts.
  for (int k = 0; k < c.K; ++k) {
    float bv = NEG;
    int be = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = j * 32 + lane;
      if (elig[j] && (s[j] > bv || (s[j] == bv && e < be))) {
        bv = s[j];
        be = e;
      }
    }
    float wv;
    int we;
    warp_argmax(bv, be, wv, we);
    sel[k] = we;
    selv[k] = wv;
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (j * 32 + lane == we) elig[j] = false;
  }
}

// Routing weights from the chosen scores, with the unfused module's rounding steps.
template <typename T>
__device__ __forceinline__ void topk_weights(const RouterCfg& c, const float (&v)[kMaxK], float (&w)[kMaxK]) {
  if (c.softmax) {
    float mx = -INFINITY;
    for (int k = 0; k < c.K; ++k) mx = fmaxf(mx, v[k]);
    float sum = 0.f;
    for (int k = 0; k < c.K; ++k) {
      w[k] = expf(v[k] - mx);
      sum += w[k];
    }
    for (int k = 0; k < c.K; ++k) w[k] = rnd<T>(w[k] / sum);
  } else if (c.norm_topk) {
    float sum = 0.f;
    for (int k = 0; k < c.K; ++k) sum += v[k];
    sum = fmaxf(rnd<T>(sum), 1e-9f);
    for (int k = 0; k < c.K; ++k) w[k] = rnd<T>(v[k] / sum);
  } else {
    for (int k = 0; k < c.K; ++k) w[k] = v[k];
  }
  for (int k = 0; k < c.K; ++k) w[k] = rnd<T>(w[k] * c.scale);
}

template <typename T>
__global__ void __launch_bounds__(256) router_fwd_kernel(const T* __restrict__ logits, RouterCfg c,
                                                         int64_t* __restrict__ idx, T* __restrict__ wout,
                                                         int* __restrict__ counts, float* __restrict__ psum) {
  const int lane = threadIdx.x & 31;
  const long nwarps = static_cast<long>(gridDim.x) * (blockDim.x >> 5);
  __shared__ float s_psum[kMaxE];
  __shared__ int s_cnt[kMaxE];
  for (int e = threadIdx.x; e < c.E; e += blockDim.x) {
    s_psum[e] = 0.f;
    s_cnt[e] = 0;
  }
  __syncthreads();
  for (long t = static_cast<long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < c.T; t += nwarps) {
    float s[kPer];
    int sel[kMaxK];
    float selv[kMaxK], w[kMaxK];
    route_token<T>(logits + t * c.E, c, lane, s, sel, selv);
    topk_weights<T>(c, selv, w);
    if (lane < c.K) {
      float wl = 0.f;
      int el = 0;
      for (int k = 0; k < c.K; ++k)
        if (k == lane) {
          wl = w[k];
          el = sel[k];
        }
      idx[t * c.K + lane] = el;
      wout[t * c.K + lane] = from_f<T>(wl);
      atomicAdd(&s_cnt[el], 1);
    }
    // aux-loss probabilities
    float norm = 1.f;
    if (!c.softmax) {
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < kPer; ++j) sum += s[j];
      norm = fmaxf(rnd<T>(warp_sum(sum)), 1e-9f);
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = j * 32 + lane;
      if (e < c.E) atomicAdd(&s_psum[e], c.softmax ? s[j] : rnd<T>(s[j] / norm));
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < c.E; e += blockDim.x) {
    if (s_cnt[e]) atomicAdd(counts + e, s_cnt[e]);
    atomicAdd(psum + e, s_psum[e]);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) router_bwd_kernel(const T* __restrict__ logits, RouterCfg c,
                                                         const int64_t* __restrict__ idx,
                                                         const T* __restrict__ dw, const float* __restrict__ dpsum,
                                                         T* __restrict__ dlogits) {
  const int lane = threadIdx.x & 31;
  const long nwarps = static_cast<long>(gridDim.x) * (blockDim.x >> 5);
  for (long t = static_cast<long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < c.T; t += nwarps) {
    const T* x = logits + t * c.E;
    // scores (same arithmetic as the forward)
    float s[kPer];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = j * 32 + lane;
      s[j] = e < c.E ? to_f(x[e]) : -INFINITY;
      mx = fmaxf(mx, s[j]);
    }
    if (c.softmax) {
      mx = warp_max(mx);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        s[j] = (j * 32 + lane) < c.E ? expf(s[j] - mx) : 0.f;
        sum += s[j];
      }
      sum = warp_sum(sum);
#pragma unroll
      for (int j = 0; j < kPer; ++j) s[j] = rnd<T>(s[j] / sum);
    } else {
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        s[j] = (j * 32 + lane) < c.E ? rnd<T>(1.f / (1.f + expf(-s[j]))) : 0.f;
    }
    // d scores from the aux loss: dn_e = dpsum[e]
    float ds[kPer];
    float S = 1.f, dot = 0.f;
    if (!c.softmax) {
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < kPer; ++j) sum += s[j];
      S = fmaxf(warp_sum(sum), 1e-9f);
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int e = j * 32 + lane;
        dot += e < c.E ? dpsum[e] * s[j] : 0.f;
      }
      dot = warp_sum(dot);
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = j * 32 + lane;
      const float dn = e < c.E ? dpsum[e] : 0.f;
      ds[j] = c.softmax ? dn : dn / S - dot / (S * S);
    }
    // d scores from the routing weights
    int sel[kMaxK];
    float v[kMaxK], g[kMaxK];
    for (int k = 0; k < c.K; ++k) {
      sel[k] = static_cast<int>(idx[t * c.K + k]);
      g[k] = to_f(dw[t * c.K + k]) * c.scale;
      const int e = sel[k];
      const int src = e & 31, jj = e >> 5;
      float mine = 0.f;
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (j == jj) mine = s[j];
      v[k] = __shfl_sync(0xffffffffu, mine, src);
    }
    float dv[kMaxK];
    if (c.softmax) {
      float mx2 = -INFINITY;
      for (int k = 0; k < c.K; ++k) mx2 = fmaxf(mx2, v[k]);
      float sum = 0.f, p[kMaxK];
      for (int k = 0; k < c.K; ++k) {
        p[k] = expf(v[k] - mx2);
        sum += p[k];
      }
      float dp = 0.f;
      for (int k = 0; k < c.K; ++k) {
        p[k] /= sum;
        dp += g[k] * p[k];
      }
      for (int k = 0; k < c.K; ++k) dv[k] = p[k] * (g[k] - dp);
    } else if (c.norm_topk) {
      float V = 0.f, gv = 0.f;
      for (int k = 0; k < c.K; ++k) {
        V += v[k];
        gv += g[k] * v[k];
      }
      V = fmaxf(V, 1e-9f);
      for (int k = 0; k < c.K; ++k) dv[k] = g[k] / V - gv / (V * V);
    } else {
      for (int k = 0; k < c.K; ++k) dv[k] = g[k];
    }
    for (int k = 0; k < c.K; ++k) {
      const int e = sel[k];
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (j * 32 + lane == e) ds[j] += dv[k];
    }
    // through the scoring function
    if (c.softmax) {
      float dot2 = 0.f;
#pragma unroll
      for (int j = 0; j < kPer; ++j) dot2 += ds[j] * s[j];
      dot2 = warp_sum(dot2);
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int e = j * 32 + lane;
        if (e < c.E) dlogits[t * c.E + e] = from_f<T>(s[j] * (ds[j] - dot2));
      }
    } else {
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int e = j * 32 + lane;
        if (e < c.E) dlogits[t * c.E + e] = from_f<T>(ds[j] * s[j] * (1.f - s[j]));
      }
    }
  }
}

RouterCfg make_cfg(const at::Tensor& logits, int64_t K, bool softmax, int64_t n_group, int64_t topk_group,
                   bool norm_topk, double scale) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.is_contiguous(), "router: logits [T, E] contiguous");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 || logits.scalar_type() == at::kFloat, "router: bf16 or fp32");
  const int64_t E = logits.size(1);
  TORCH_CHECK(E >= 1 && E <= kMaxE, "router: at most ", kMaxE, " experts");
  TORCH_CHECK(K >= 1 && K <= kMaxK && K <= E, "router: top-k in [1, 8]");
  TORCH_CHECK(n_group >= 1 && n_group <= kMaxGroups && E % n_group == 0 && topk_group >= 1 && topk_group <= n_group,
              "router: bad group routing parameters");
  RouterCfg c{};
  c.T = static_cast<int>(logits.size(0));
  c.E = static_cast<int>(E);
  c.K = static_cast<int>(K);
  c.softmax = softmax ? 1 : 0;
  c.n_group = static_cast<int>(n_group);
  c.topk_group = static_cast<int>(topk_group);
  c.norm_topk = norm_topk ? 1 : 0;
  c.scale = static_cast<float>(scale);
  return c;
}

int router_grid(int dev, int T) {
  const int want = (T + 7) / 8;
  return std::max(1, std::min(want, num_sms(dev) * 4));
}

}  // namespace

// Returns (topk_idx int64 [T, K], topk_w [T, K] logits dtype, counts int32 [E], psum fp32 [E]).
std::vector<at::Tensor> router_fwd(const at::Tensor& logits, int64_t K, bool softmax, int64_t n_group,
                                   int64_t topk_group, bool norm_topk, double scale) {
  RouterCfg c = make_cfg(logits, K, softmax, n_group, topk_group, norm_topk, scale);
  auto idx = at::empty({c.T, c.K}, logits.options().dtype(at::kLong));
  auto w = at::empty({c.T, c.K}, logits.options());
  auto counts = at::zeros({c.E}, logits.options().dtype(at::kInt));
  auto psum = at::zeros({c.E}, logits.options().dtype(at::kFloat));
  if (c.T == 0) return {idx, w, counts, psum};
  const int dev = logits.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  if (logits.scalar_type() == at::kBFloat16)
    router_fwd_kernel<bf16><<<router_grid(dev, c.T), 256, 0, stream>>>(
        reinterpret_cast<const bf16*>(logits.data_ptr()), c, idx.data_ptr<int64_t>(),
        reinterpret_cast<bf16*>(w.data_ptr()), counts.data_ptr<int>(), psum.data_ptr<float>());
  else
    router_fwd_kernel<float><<<router_grid(dev, c.T), 256, 0, stream>>>(
        logits.data_ptr<float>(), c, idx.data_ptr<int64_t>(), w.data_ptr<float>(), counts.data_ptr<int>(),
        psum.data_ptr<float>());
  NTB_LAUNCH_CHECK(1);
  return {idx, w, counts, psum};
}

at::Tensor router_bwd(const at::Tensor& logits, const at::Tensor& idx, const at::Tensor& dw, const at::Tensor& dpsum,
                      int64_t K, bool softmax, int64_t n_group, int64_t topk_group, bool norm_topk, double scale) {
  RouterCfg c = make_cfg(logits, K, softmax, n_group, topk_group, norm_topk, scale);
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous() && idx.numel() == static_cast<int64_t>(c.T) * c.K,
              "router_bwd: idx int64 [T, K]");
  TORCH_CHECK(dw.scalar_type() == logits.scalar_type() && dw.is_contiguous() && dw.numel() == idx.numel(),
              "router_bwd: dw [T, K] in the logits dtype");
  TORCH_CHECK(dpsum.scalar_type() == at::kFloat && dpsum.is_contiguous() && dpsum.numel() == c.E,
              "router_bwd: dpsum fp32 [E]");
  auto dl = at::empty_like(logits);
  if (c.T == 0) return dl;
  const int dev = logits.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  if (logits.scalar_type() == at::kBFloat16)
    router_bwd_kernel<bf16><<<router_grid(dev, c.T), 256, 0, stream>>>(
        reinterpret_cast<const bf16*>(logits.data_ptr()), c, idx.data_ptr<int64_t>(),
        reinterpret_cast<const bf16*>(dw.data_ptr()), dpsum.data_ptr<float>(), reinterpret_cast<bf16*>(dl.data_ptr()));
  else
    router_bwd_kernel<float><<<router_grid(dev, c.T), 256, 0, stream>>>(
        logits.data_ptr<float>(), c, idx.data_ptr<int64_t>(), dw.data_ptr<float>(), dpsum.data_ptr<float>(),
        dl.data_ptr<float>());
  NTB_LAUNCH_CHECK(1);
  return dl;
}

}  // namespace ntb
