// Memory-bound sm_100a kernels: norms, RoPE, activations, cross-entropy,
// embedding, fused AdamW and gradient unscale/finite/norm.
//
// All are row- or element-parallel with 16-byte vector access where the
// shape allows; fp32 math internally, bf16 or fp32 storage.
//
// Reference parity (behaviour, not code):
//   RMSNorm          src/models/deepseek.py:386-438
//   LayerNorm        src/layers.py:639-781
//   RoPE (both)      src/models/deepseek.py:517-543 (interleaved rotate, half-split cache)
//   SwiGLU / GELU    src/models/moe.py:146-193, src/layers.py:1017-1095
//   cross-entropy    src/losses.py:95-133, examples/train_4d.py:725-730
//   embedding        src/layers.py:788-900
//   AdamW            src/runtime/optimizer_runtime.py:68-116, src/distributed/zero.py:451-474
//   unscale/finite   src/runtime/mixed_precision.py:813-854
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"
#include "no_alloc.h"

#include <atomic>
#include <cstdio>
#include <mutex>

namespace ntb {

using bf16 = __nv_bfloat16;

// Typed raw pointer of a tensor (bf16 tensors are viewed as __nv_bfloat16).
template <typename T>
static inline T* P(const at::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<bf16>(bf16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16(v); }

// Vector of 8 elements <-> 8 floats.
template <typename T>
__device__ __forceinline__ void ld8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void ld8<bf16>(const bf16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
  v[4] = bf16_lo(u.z); v[5] = bf16_hi(u.z); v[6] = bf16_lo(u.w); v[7] = bf16_hi(u.w);
}
template <>
__device__ __forceinline__ void ld8<float>(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename T>
__device__ __forceinline__ void st8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void st8<bf16>(bf16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]); u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]); u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void st8<float>(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Block-wide sum over up to 1024 threads (result broadcast to every thread).
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (w == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : -INFINITY;
  if (w == 0) t = warp_max(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

static int row_threads(int64_t H) {
  int t = 32;
  while (t < 1024 && t * 8 < H) t *= 2;
  return t;
}

#define NTB_DISPATCH_FLOAT(T_, NAME, ...)                                   \
  [&] {                                                                     \
    if ((T_) == at::kBFloat16) {                                            \
      using scalar_t = bf16;                                                \
      return __VA_ARGS__();                                                 \
    } else if ((T_) == at::kFloat) {                                        \
      using scalar_t = float;                                               \
      return __VA_ARGS__();                                                 \
    } else {                                                                \
      TORCH_CHECK(false, NAME, ": unsupported dtype ", (T_));              \
    }                                                                       \
  }()

// =========================================================== RMSNorm
// h = x (+ residual); y = h * rsqrt(mean(h^2) + eps) * w.
template <typename T, bool VEC>
__global__ void rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ res, const T* __restrict__ w,
                                   T* __restrict__ y, T* __restrict__ h_out, float* __restrict__ rstd_out, int H,
                                   float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * H;
  const T* rr = res ? res + row * H : nullptr;
  float ss = 0.f;
  if (VEC) {
    for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
      float v[8];
      ld8(xr + i, v);
      if (rr) {
        float r[8];
        ld8(rr + i, r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] += r[j];
        st8(h_out + row * H + i, v);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
    }
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      float v = to_f(xr[i]);
      if (rr) {
        v += to_f(rr[i]);
        h_out[row * H + i] = from_f<T>(v);
      }
      ss += v * v;
    }
  }
  ss = block_sum(ss, red);
  const float rstd = rsqrtf(ss / H + eps);
  if (threadIdx.x == 0) rstd_out[row] = rstd;
  const T* hr = rr ? h_out + row * H : xr;
  if (VEC) {
    for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
      float v[8], g[8];
      ld8(hr + i, v);
      ld8(w + i, g);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = v[j] * rstd * g[j];
      st8(y + row * H + i, v);
    }
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) y[row * H + i] = from_f<T>(to_f(hr[i]) * rstd * to_f(w[i]));
  }
}

// dx = rstd * (g - n * mean(g * n)), g = dy * w, n = h * rstd; dw partials per block.
// Scalar form, for rows whose width or pointers do not allow 16-byte vectors.
template <typename T>
__global__ void rmsnorm_bwd_scalar_kernel(const T* __restrict__ dy, const T* __restrict__ h, const T* __restrict__ w,
                                          const float* __restrict__ rstd, const T* __restrict__ dres,
                                          T* __restrict__ dx, float* __restrict__ dw_part, int64_t rows, int H,
                                          int rows_per_block) {
  __shared__ float red[32];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  float* dwp = dw_part + static_cast<int64_t>(blockIdx.x) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) dwp[i] = 0.f;
  for (int64_t row = r0; row < r0 + rows_per_block && row < rows; ++row) {
    const float rs = rstd[row];
    const T* dyr = dy + row * H;
    const T* hr = h + row * H;
    float dot = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) dot += to_f(dyr[i]) * to_f(w[i]) * to_f(hr[i]);
    dot = block_sum(dot, red);
    const float mean_gn = dot * rs / H;  // mean(g * n)
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const float a = to_f(dyr[i]), n = to_f(hr[i]) * rs;
      float o = rs * (a * to_f(w[i]) - n * mean_gn);
      if (dres) o += to_f(dres[row * H + i]);
      dx[row * H + i] = from_f<T>(o);
      dwp[i] += a * n;
    }
  }
}

// Vector form. A CTA owns a contiguous run of rows and streams them through a ring of shared-memory
// stages filled by the TMA engine (one 1-D bulk copy per source row: dy, h and, when given, dres),
// so several rows are in flight per CTA without holding them in registers. Each thread owns NCH
// chunks of 8 columns, the same ones for every row, so its dW contribution stays in registers
// for the whole run and is written once, as this CTA's partial row.
// Per row there is exactly one CTA barrier. Before it, each thread reads its slice of the stage
// (dot product g*h with g = dy*w, and the dW update, which needs no reduction); the barrier
// completes the reduction; after it the thread reads the slice again and writes
// dx = rs*g - c2*h (+ dres), c2 = rs^3 * mean(g*h). Row i's barrier also proves that every thread
// finished row i-1, so that stage is refilled then (stages - 1 rows stay in flight ahead).
// Every mbarrier wait is bounded; on a timeout (status raised) the CTA waits, again bounded, for
// the copies it issued and returns without writing its partial.
template <typename T, int NCH, bool RES>
__global__ void __launch_bounds__(512, 1) rmsnorm_bwd_ring_kernel(
    const T* __restrict__ dy, const T* __restrict__ h, const T* __restrict__ w, const float* __restrict__ rstd,
    const T* __restrict__ dres, T* __restrict__ dx, float* __restrict__ dw_part, int64_t rows, int H,
    int rows_per_block, int stages, int* status) {
  extern __shared__ __align__(128) uint8_t ring_smem[];
  __shared__ uint64_t full[8];
  __shared__ __align__(16) float red[2][16];
  constexpr int kSrc = RES ? 3 : 2;
  const uint32_t row_bytes = static_cast<uint32_t>(H) * sizeof(T);
  T* ring = reinterpret_cast<T*>(ring_smem);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t r_end = rows < r0 + rows_per_block ? rows : r0 + rows_per_block;
  const int n = r_end > r0 ? static_cast<int>(r_end - r0) : 0;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nw4 = (blockDim.x + 127) >> 7;  // float4 groups of warp partials (blockDim <= 512: <= 4)
  if (tid == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  if (tid < 32) red[tid >> 4][tid & 15] = 0.f;  // unused warp slots read as zero
  __syncthreads();
  int issued = 0;  // rows whose copies were issued (thread 0 only)
  auto issue_next = [&]() {
    const int slot = issued % stages;
    const int64_t row = r0 + issued;
    mbar_expect_tx(&full[slot], kSrc * row_bytes);
    T* base = ring + static_cast<int64_t>(slot) * kSrc * H;
    bulk_load_1d(base, dy + row * H, row_bytes, &full[slot]);
    bulk_load_1d(base + H, h + row * H, row_bytes, &full[slot]);
    if (RES) bulk_load_1d(base + 2 * H, dres + row * H, row_bytes, &full[slot]);
    ++issued;
  };
  if (tid == 0)
    while (issued < stages && issued < n) issue_next();
  float wv[NCH][8], dwa[NCH][8];
  bool act[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * blockDim.x + tid) * 8;
    act[c] = col < H;
#pragma unroll
    for (int j = 0; j < 8; ++j) dwa[c][j] = wv[c][j] = 0.f;
    if (act[c]) ld8(w + col, wv[c]);
  }
  const float inv_h = 1.f / static_cast<float>(H);
  bool failed = false;
  int i = 0;
  for (; i < n; ++i) {
    const int slot = i % stages;
    const uint32_t parity = static_cast<uint32_t>(i / stages) & 1u;
    const int64_t row = r0 + i;
    const float rs = rstd[row];
    const bool ok = mbar_wait(&full[slot], parity, status, kStatusTimeoutProducer);
    const T* base = ring + static_cast<int64_t>(slot) * kSrc * H;
    float dot = 0.f;
    if (ok) {
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        if (!act[c]) continue;
        const int col = (c * blockDim.x + tid) * 8;
        float a[8], b[8];
        ld8(base + col, a);
        ld8(base + H + col, b);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          dot = fmaf(a[j] * wv[c][j], b[j], dot);
          dwa[c][j] = fmaf(a[j] * rs, b[j], dwa[c][j]);
        }
      }
    }
    dot = warp_sum(dot);
    if (lane == 0) red[i & 1][wid] = dot;
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    // Every thread is past row i-1: its stage takes the next row.
    if (tid == 0 && i >= 1 && issued < n) issue_next();
    float tot = 0.f;
    for (int k = 0; k < nw4; ++k) {
      const float4 q = reinterpret_cast<const float4*>(red[i & 1])[k];
      tot += (q.x + q.y) + (q.z + q.w);
    }
    const float c2 = rs * rs * rs * tot * inv_h;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      if (!act[c]) continue;
      const int col = (c * blockDim.x + tid) * 8;
      float a[8], b[8], d[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, o[8];
      ld8(base + col, a);
      ld8(base + H + col, b);
      if (RES) ld8(base + 2 * H + col, d);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = fmaf(-c2, b[j], fmaf(rs, a[j] * wv[c][j], d[j]));
      st8(dx + row * H + col, o);
    }
  }
  if (failed) {
    // Drain: wait (bounded) for every copy issued and not consumed, then return.
    if (tid == 0) {
      for (int k = i; k < issued; ++k) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[k % stages], static_cast<uint32_t>(k / stages) & 1u) &&
               globaltimer_ns() - t0 < NTB_WAIT_LIMIT_NS) {
        }
      }
    }
    __syncthreads();
    return;
  }
  float* dwp = dw_part + static_cast<int64_t>(blockIdx.x) * H;
#pragma unroll
  for (int c = 0; c < NCH; ++c)
    if (act[c]) st8(dwp + (c * blockDim.x + tid) * 8, dwa[c]);
}

// out[i] (+)= sum over p of part[p, i], in a fixed order (deterministic for a given partial count).
// A CTA covers 32 columns with 8 warps: lane = column, warps stride over the partial rows with four
// loads in flight each, then the 8 warp sums are added in warp order. OutT is the stored type of
// the result (the weight's dtype, or fp32); ACC adds into `out` (an fp32 gradient bucket).
template <typename OutT, bool ACC>
__global__ void __launch_bounds__(256) colsum_kernel(const float* __restrict__ part, int nparts, int H,
                                                     OutT* __restrict__ out) {
  __shared__ float acc_s[8][33];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (col < H) {
    int p = wid;
    for (; p + 24 < nparts; p += 32) {
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] += part[static_cast<int64_t>(p + 8 * u) * H + col];
    }
    for (int u = 0; p < nparts; p += 8, ++u) acc[u & 3] += part[static_cast<int64_t>(p) * H + col];
  }
  acc_s[wid][lane] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  __syncthreads();
  if (wid == 0 && col < H) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += acc_s[k][lane];
    if (ACC) t += to_f(out[col]);
    out[col] = from_f<OutT>(t);
  }
}

// Launch plan of the RMSNorm backward for `rows` x H: vector ring kernel when H % 8 == 0 and every
// pointer is 16-byte aligned, else the scalar kernel. `max_parts` bounds the number of CTAs (one
// partial row of `part` each). Returns the number of partial rows written, which colsum reduces.
struct RmsBwdPlan {
  bool ring = false;
  int nch = 1, threads = 32, blocks = 1, rows_per_block = 1, stages = 2;
  size_t smem = 0;
};

static RmsBwdPlan plan_rmsnorm_bwd(int64_t rows, int H, int elem_bytes, bool vec, bool res, int nsm, int max_parts) {
  RmsBwdPlan p;
  const int k_src = res ? 3 : 2;
  const size_t stage_bytes = static_cast<size_t>(k_src) * H * elem_bytes;
  const int chunks = (H + 7) / 8;
  // Two 8-column chunks per thread (one when the row is narrow), at most 512 threads: the per-row
  // cost (barrier, wait, cross-warp sum) is shared by 16 columns. Rows up to 8192 wide.
  p.threads = std::min(512, ((chunks + 1) / 2 + 31) / 32 * 32);
  p.nch = (chunks + p.threads - 1) / p.threads;
  // Ring: at least two stages in the 200 KB a CTA may use, at most four.
  const int fit = static_cast<int>(std::min<size_t>(4, (200u * 1024u) / std::max<size_t>(stage_bytes, 1)));
  p.ring = vec && H % 8 == 0 && p.nch <= 2 && fit >= 2;
  if (p.ring) {
    p.stages = fit;
    p.smem = p.stages * stage_bytes;
    // Up to three CTAs per SM, as shared memory (about 220 KB usable) allows.
    const int per_sm = static_cast<int>(std::max<size_t>(1, std::min<size_t>(3, (220u * 1024u) / p.smem)));
    p.blocks = static_cast<int>(std::min<int64_t>({rows, static_cast<int64_t>(nsm) * per_sm,
                                                   static_cast<int64_t>(max_parts)}));
  } else {
    p.threads = row_threads(H);
    p.nch = 1;
    p.blocks = static_cast<int>(std::min<int64_t>({rows, static_cast<int64_t>(nsm) * 4,
                                                   static_cast<int64_t>(max_parts)}));
  }
  p.blocks = std::max(p.blocks, 1);
  p.rows_per_block = static_cast<int>((rows + p.blocks - 1) / p.blocks);
  return p;
}

template <typename T, int NCH, bool RES>
static cudaError_t launch_ring(const RmsBwdPlan& p, const T* dy, const T* h, const T* w, const float* rstd,
                               const T* dres, T* dx, float* part, int64_t rows, int H, int* status,
                               cudaStream_t stream) {
  auto kern = rmsnorm_bwd_ring_kernel<T, NCH, RES>;
  // The dynamic shared-memory limit is raised once per device to the largest size seen so far.
  static std::atomic<int> smem_set[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::atomic<int>& cur = smem_set[dev & 63];
  if (cur.load() < static_cast<int>(p.smem)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(p.smem));
    if (e != cudaSuccess) return e;
    cur.store(static_cast<int>(p.smem));
  }
  kern<<<p.blocks, p.threads, p.smem, stream>>>(dy, h, w, rstd, dres, dx, part, rows, H, p.rows_per_block, p.stages,
                                                status);
  return cudaSuccess;
}

// Queues the two kernels of the RMSNorm backward (the per-CTA pass writing `part`, then the column
// sum) and returns the first CUDA error of the set-up or launches. The column sum stores dW as T in
// `dw_t`, or as fp32 in `dw_f32` (added to its contents when `accumulate`); exactly one is given.
template <typename T>
static cudaError_t launch_rmsnorm_bwd(const T* dy, const T* h, const T* w, const float* rstd, const T* dres, T* dx,
                                      float* part, T* dw_t, float* dw_f32, bool accumulate, int64_t rows, int H,
                                      bool vec, int nsm, int max_parts, int* status, cudaStream_t stream) {
  const RmsBwdPlan p = plan_rmsnorm_bwd(rows, H, sizeof(T), vec, dres != nullptr, nsm, max_parts);
  cudaError_t e = cudaSuccess;
  if (p.ring) {
    const bool r = dres != nullptr;
    if (p.nch == 1) e = r ? launch_ring<T, 1, true>(p, dy, h, w, rstd, dres, dx, part, rows, H, status, stream)
                          : launch_ring<T, 1, false>(p, dy, h, w, rstd, dres, dx, part, rows, H, status, stream);
    else e = r ? launch_ring<T, 2, true>(p, dy, h, w, rstd, dres, dx, part, rows, H, status, stream)
               : launch_ring<T, 2, false>(p, dy, h, w, rstd, dres, dx, part, rows, H, status, stream);
  } else {
    rmsnorm_bwd_scalar_kernel<T><<<p.blocks, p.threads, 0, stream>>>(dy, h, w, rstd, dres, dx, part, rows, H,
                                                                     p.rows_per_block);
  }
  if (e != cudaSuccess) return e;
  const int grid = (H + 31) / 32;
  if (dw_f32 && accumulate) colsum_kernel<float, true><<<grid, 256, 0, stream>>>(part, p.blocks, H, dw_f32);
  else if (dw_f32) colsum_kernel<float, false><<<grid, 256, 0, stream>>>(part, p.blocks, H, dw_f32);
  else colsum_kernel<T, false><<<grid, 256, 0, stream>>>(part, p.blocks, H, dw_t);
  return cudaGetLastError();
}

static bool vec8_ok(const at::Tensor& t, int64_t H) {
  return H % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0;
}

std::vector<at::Tensor> rmsnorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& residual,
                                    const at::Tensor& w, double eps) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && w.is_contiguous(), "rmsnorm_fwd: contiguous CUDA tensors");
  const int64_t H = x.size(-1);
  const int64_t rows = x.numel() / H;
  TORCH_CHECK(w.numel() == H && w.scalar_type() == x.scalar_type(), "rmsnorm_fwd: weight");
  auto y = at::empty_like(x);
  at::Tensor h;
  const bool has_res = residual.has_value();
  if (has_res) {
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == x.sizes(), "rmsnorm_fwd: residual");
    h = at::empty_like(x);
  }
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  if (rows == 0) return {y, h.defined() ? h : x, rstd};
  auto stream = at::cuda::getCurrentCUDAStream();
  const int threads = row_threads(H);
  bool vec = vec8_ok(x, H) && vec8_ok(w, H) && vec8_ok(y, H);
  if (has_res) vec = vec && vec8_ok(*residual, H) && vec8_ok(h, H);
  NTB_DISPATCH_FLOAT(x.scalar_type(), "rmsnorm_fwd", [&] {
    const scalar_t* rp = has_res ? P<scalar_t>(*residual) : nullptr;
    scalar_t* hp = has_res ? P<scalar_t>(h) : nullptr;
    if (vec)
      rmsnorm_fwd_kernel<scalar_t, true><<<rows, threads, 0, stream>>>(P<scalar_t>(x), rp, P<scalar_t>(w),
                                                                       P<scalar_t>(y), hp, rstd.data_ptr<float>(), H, eps);
    else
      rmsnorm_fwd_kernel<scalar_t, false><<<rows, threads, 0, stream>>>(P<scalar_t>(x), rp, P<scalar_t>(w),
                                                                        P<scalar_t>(y), hp, rstd.data_ptr<float>(), H, eps);
  });
  NTB_LAUNCH_CHECK(1);
  return {y, has_res ? h : x, rstd};
}

// Returns (dx, dw). dres (optional) is added into dx (gradient flowing along the residual stream).
// With dw_into (an fp32 tensor of H elements, e.g. the weight's main_grad view of a gradient bucket)
// the weight gradient is added into it and the returned dw is undefined (None in Python).
std::vector<at::Tensor> rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& h, const at::Tensor& w,
                                    const at::Tensor& rstd, const c10::optional<at::Tensor>& dres,
                                    const c10::optional<at::Tensor>& dw_into) {
  TORCH_CHECK(dy.is_contiguous() && h.is_contiguous(), "rmsnorm_bwd: contiguous");
  const int64_t H = h.size(-1);
  const int64_t rows = h.numel() / H;
  const bool into = dw_into.has_value();
  if (into)
    TORCH_CHECK(dw_into->is_cuda() && dw_into->scalar_type() == at::kFloat && dw_into->is_contiguous() &&
                    dw_into->numel() == H,
                "rmsnorm_bwd: dw_into must be a contiguous fp32 CUDA tensor of H elements");
  auto dx = at::empty_like(h);
  at::Tensor dw = into ? at::Tensor() : at::empty({H}, w.options());
  if (rows == 0) {
    if (!into) dw.zero_();
    return {dx, dw};
  }
  const int dev = h.get_device();
  const int nsm = num_sms(dev);
  bool vec = vec8_ok(dy, H) && vec8_ok(h, H) && vec8_ok(w, H) && vec8_ok(dx, H);
  if (dres.has_value()) vec = vec && vec8_ok(*dres, H);
  const int max_parts = 8 * nsm;
  const RmsBwdPlan plan = plan_rmsnorm_bwd(rows, static_cast<int>(H), h.element_size(), vec, dres.has_value(), nsm,
                                           max_parts);
  auto part = at::empty({plan.blocks, H}, h.options().dtype(at::kFloat));
  auto stream = at::cuda::getCurrentCUDAStream();
  cudaError_t e = cudaSuccess;
  NTB_DISPATCH_FLOAT(h.scalar_type(), "rmsnorm_bwd", [&] {
    TORCH_CHECK(w.scalar_type() == h.scalar_type(), "rmsnorm_bwd: weight dtype");
    const scalar_t* dr = dres.has_value() ? P<scalar_t>(*dres) : nullptr;
    e = launch_rmsnorm_bwd<scalar_t>(P<scalar_t>(dy), P<scalar_t>(h), P<scalar_t>(w), rstd.data_ptr<float>(), dr,
                                     P<scalar_t>(dx), part.data_ptr<float>(), into ? nullptr : P<scalar_t>(dw),
                                     into ? dw_into->data_ptr<float>() : nullptr, into, rows, static_cast<int>(H),
                                     vec, nsm, max_parts, device_status(dev), stream);
  });
  note_launches(2);
  NTB_CUDA_CHECK(e);
  return {dx, dw};
}

// ----------------------------------------------------------- allocation-free RMSNorm backward
// Variant of rmsnorm_bwd for callers that cannot allocate (see no_alloc.h): the same kernels and
// launch plan, with the per-CTA dW partials in a file-scope device array instead of a per-call
// tensor, and at most kNoAllocBlocks CTAs. Each CTA overwrites its whole partial row, so the array
// needs no initialisation.
constexpr int kNoAllocBlocks = 128;
static __device__ __align__(256) float g_rmsnorm_bwd_scratch[kNoAllocBlocks * NTB_NOALLOC_RMSNORM_MAX_H];

constexpr int kNoAllocMaxDevices = 64;
struct NoAllocSetup {
  unsigned long long ctx_id = 0;  // cuCtxGetId of the context the address was resolved in (0: none)
  float* scratch = nullptr;
  int nsm = 0;
};
static NoAllocSetup g_noalloc_setup[kNoAllocMaxDevices];
static std::mutex g_noalloc_mu;
static thread_local char g_noalloc_err[256] = "";

static int noalloc_fail(int code, const char* what, cudaError_t e) {
  if (e != cudaSuccess)
    std::snprintf(g_noalloc_err, sizeof(g_noalloc_err), "%s: %s", what, cudaGetErrorString(e));
  else
    std::snprintf(g_noalloc_err, sizeof(g_noalloc_err), "%s", what);
  return code;
}

// Id of the current context (unique for the process's lifetime, unlike the handle), through the
// driver entry point so that the extension does not link against libcuda directly.
static cudaError_t current_context_id(unsigned long long* id) {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  if (!get_current || !get_id) {
    void* f1 = nullptr;
    void* f2 = nullptr;
    cudaDriverEntryPointQueryResult q1, q2;
    cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1);
    if (e != cudaSuccess || q1 != cudaDriverEntryPointSuccess) return e != cudaSuccess ? e : cudaErrorNotSupported;
    e = cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2);
    if (e != cudaSuccess || q2 != cudaDriverEntryPointSuccess) return e != cudaSuccess ? e : cudaErrorNotSupported;
    get_current = reinterpret_cast<GetCurrent>(f1);
    get_id = reinterpret_cast<GetId>(f2);
  }
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return cudaErrorDeviceUninitialized;
  return get_id(ctx, id) == CUDA_SUCCESS ? cudaSuccess : cudaErrorDeviceUninitialized;
}

}  // namespace ntb

extern "C" __attribute__((visibility("default"))) const char* ntb_noalloc_last_error(void) {
  return ntb::g_noalloc_err;
}

extern "C" __attribute__((visibility("default"))) int ntb_rmsnorm_bwd_bf16_noalloc(
    const void* dy, const void* h, const void* w, const float* rstd, const void* dres, void* dx, float* dw,
    int64_t rows, int H, cudaStream_t stream) {
  using namespace ntb;
  using T = __nv_bfloat16;
  if (H < 1 || H > NTB_NOALLOC_RMSNORM_MAX_H || rows < 0) {
    std::snprintf(g_noalloc_err, sizeof(g_noalloc_err),
                  "ntb_rmsnorm_bwd_bf16_noalloc: H=%d rows=%lld outside H in [1, %d], rows >= 0", H,
                  static_cast<long long>(rows), NTB_NOALLOC_RMSNORM_MAX_H);
    return 1;
  }
  // An error left by earlier work on this thread is reported as such and left pending for its owner.
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) return noalloc_fail(3, "an earlier CUDA error is pending (not cleared)", e);
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(2, "cudaGetDevice", e);
  if (dev < 0 || dev >= kNoAllocMaxDevices) return noalloc_fail(2, "device index beyond the set-up table", cudaSuccess);
  unsigned long long ctx_id = 0;
  e = current_context_id(&ctx_id);
  if (e != cudaSuccess) return noalloc_fail(2, "cuCtxGetCurrent / cuCtxGetId", e);
  NoAllocSetup setup;
  {
    // Set-up per device and context, with that device current: resolve the scratch array's
    // address. A new context on the device (after cudaDeviceReset, say) resolves it again.
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocSetup& s = g_noalloc_setup[dev];
    if (s.ctx_id != ctx_id || s.scratch == nullptr) {
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_rmsnorm_bwd_scratch);
      if (e != cudaSuccess) return noalloc_fail(2, "cudaGetSymbolAddress(scratch)", e);
      int nsm = 0;
      e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return noalloc_fail(2, "cudaDeviceGetAttribute(SM count)", e);
      s.scratch = static_cast<float*>(ptr);
      s.nsm = nsm;
      s.ctx_id = ctx_id;
    }
    setup = s;
  }
  g_noalloc_err[0] = '\0';
  if (rows == 0) return 0;
  const bool vec = (H % 8 == 0) && ((reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(h) |
                                     reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(dx) |
                                     (dres ? reinterpret_cast<uintptr_t>(dres) : 0)) &
                                    15) == 0;
  e = launch_rmsnorm_bwd<T>(static_cast<const T*>(dy), static_cast<const T*>(h), static_cast<const T*>(w), rstd,
                            static_cast<const T*>(dres), static_cast<T*>(dx), setup.scratch, nullptr, dw, false, rows,
                            H, vec, setup.nsm, kNoAllocBlocks, nullptr, stream);
  if (e != cudaSuccess) return noalloc_fail(2, "kernel launch", e);
  return 0;
}

namespace ntb {

// =========================================================== LayerNorm
template <typename T>
__global__ void layernorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
                                     T* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                     int H, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * H;
  float s = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) s += to_f(xr[i]);
  const float mean = block_sum(s, red) / H;
  float v = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float d = to_f(xr[i]) - mean;
    v += d * d;
  }
  const float var = block_sum(v, red) / H;
  const float rstd = rsqrtf(var + eps);
  if (threadIdx.x == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float o = (to_f(xr[i]) - mean) * rstd * to_f(w[i]);
    if (b) o += to_f(b[i]);
    y[row * H + i] = from_f<T>(o);
  }
}

template <typename T>
__global__ void layernorm_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x, const T* __restrict__ w,
                                     const float* __restrict__ mean, const float* __restrict__ rstd,
                                     T* __restrict__ dx, float* __restrict__ dw_part, float* __restrict__ db_part,
                                     int64_t rows, int H, int rows_per_block) {
  __shared__ float red[32];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  float* dwp = dw_part + static_cast<int64_t>(blockIdx.x) * H;
  float* dbp = db_part + static_cast<int64_t>(blockIdx.x) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    dwp[i] = 0.f;
    dbp[i] = 0.f;
  }
  for (int64_t row = r0; row < r0 + rows_per_block && row < rows; ++row) {
    const float mu = mean[row], rs = rstd[row];
    float a = 0.f, bsum = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const float g = to_f(dy[row * H + i]) * to_f(w[i]);
      const float xh = (to_f(x[row * H + i]) - mu) * rs;
      a += g;
      bsum += g * xh;
    }
    a = block_sum(a, red) / H;
    bsum = block_sum(bsum, red) / H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const float d = to_f(dy[row * H + i]);
      const float g = d * to_f(w[i]);
      const float xh = (to_f(x[row * H + i]) - mu) * rs;
      dx[row * H + i] = from_f<T>(rs * (g - a - xh * bsum));
      dwp[i] += d * xh;
      dbp[i] += d;
    }
  }
}

std::vector<at::Tensor> layernorm_fwd(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& b,
                                      double eps) {
  TORCH_CHECK(x.is_contiguous(), "layernorm_fwd: contiguous");
  const int64_t H = x.size(-1), rows = x.numel() / H;
  auto y = at::empty_like(x);
  auto mean = at::empty({rows}, x.options().dtype(at::kFloat));
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  if (rows == 0) return {y, mean, rstd};
  auto stream = at::cuda::getCurrentCUDAStream();
  NTB_DISPATCH_FLOAT(x.scalar_type(), "layernorm_fwd", [&] {
    layernorm_fwd_kernel<scalar_t><<<rows, row_threads(H), 0, stream>>>(
        P<scalar_t>(x), P<scalar_t>(w), b.has_value() ? P<scalar_t>(*b) : nullptr,
        P<scalar_t>(y), mean.data_ptr<float>(), rstd.data_ptr<float>(), H, eps);
  });
  NTB_LAUNCH_CHECK(1);
  return {y, mean, rstd};
}

std::vector<at::Tensor> layernorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                      const at::Tensor& mean, const at::Tensor& rstd) {
  const int64_t H = x.size(-1), rows = x.numel() / H;
  auto dx = at::empty_like(x);
  auto dw = at::zeros({H}, x.options().dtype(at::kFloat));
  auto db = at::zeros({H}, x.options().dtype(at::kFloat));
  if (rows == 0) return {dx, dw.to(w.scalar_type()), db.to(w.scalar_type())};
  const int blocks = static_cast<int>(std::min<int64_t>(rows, num_sms(x.get_device()) * 4));
  const int rpb = static_cast<int>((rows + blocks - 1) / blocks);
  auto pw = at::empty({blocks, H}, x.options().dtype(at::kFloat));
  auto pb = at::empty({blocks, H}, x.options().dtype(at::kFloat));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto dyc = dy.contiguous();
  NTB_DISPATCH_FLOAT(x.scalar_type(), "layernorm_bwd", [&] {
    layernorm_bwd_kernel<scalar_t><<<blocks, row_threads(H), 0, stream>>>(
        P<scalar_t>(dyc), P<scalar_t>(x), P<scalar_t>(w), mean.data_ptr<float>(),
        rstd.data_ptr<float>(), P<scalar_t>(dx), pw.data_ptr<float>(), pb.data_ptr<float>(), rows, H, rpb);
  });
  colsum_kernel<float, false><<<(H + 31) / 32, 256, 0, stream>>>(pw.data_ptr<float>(), blocks, H,
                                                                  dw.data_ptr<float>());
  colsum_kernel<float, false><<<(H + 31) / 32, 256, 0, stream>>>(pb.data_ptr<float>(), blocks, H,
                                                                  db.data_ptr<float>());
  NTB_LAUNCH_CHECK(3);
  return {dx, dw.to(w.scalar_type()), db.to(w.scalar_type())};
}

// =========================================================== RoPE
// x: [T, heads, D] view with row stride (elements) `sx` between tokens and
// `sh` between heads; rotary part occupies columns [off, off + R).
// mode 0 (half-split, Llama/NeoX): pairs (i, i + R/2), angle pos * f[i].
// mode 1 (interleaved pairs with half-split cache): element j of the pair
//   (2i, 2i+1) uses angle pos * f[j mod R/2]; out[2i] = x[2i] c[2i] - x[2i+1] s[2i],
//   out[2i+1] = x[2i+1] c[2i+1] + x[2i] s[2i+1] (matches the reference's
//   rotate_half over interleaved elements combined with cat(freqs, freqs)).
// inverse=true applies the transpose (backward).
template <typename T>
__global__ void rope_kernel(T* __restrict__ x, const int64_t* __restrict__ pos, int T_, int heads, int64_t sx,
                            int64_t sh, int off, int R, int seq_len, float theta, int mode, bool inverse) {
  const int half = R / 2;
  const int64_t total = static_cast<int64_t>(T_) * heads * half;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = idx % half;
    const int64_t th = idx / half;
    const int hd = th % heads;
    const int t = th / heads;
    const float p = pos ? static_cast<float>(pos[t]) : static_cast<float>(t % seq_len);
    T* base = x + t * sx + hd * sh + off;
    if (mode == 0) {
      const float f = powf(theta, -2.f * i / R);
      float s, c;
      sincosf(p * f, &s, &c);
      if (inverse) s = -s;
      const float a = to_f(base[i]), b = to_f(base[i + half]);
      base[i] = from_f<T>(a * c - b * s);
      base[i + half] = from_f<T>(b * c + a * s);
    } else {
      const int j0 = 2 * i, j1 = 2 * i + 1;
      const float f0 = powf(theta, -2.f * (j0 % half) / R);
      const float f1 = powf(theta, -2.f * (j1 % half) / R);
      float s0, c0, s1, c1;
      sincosf(p * f0, &s0, &c0);
      sincosf(p * f1, &s1, &c1);
      const float a = to_f(base[j0]), b = to_f(base[j1]);
      if (!inverse) {
        base[j0] = from_f<T>(a * c0 - b * s0);
        base[j1] = from_f<T>(b * c1 + a * s1);
      } else {
        base[j0] = from_f<T>(a * c0 + b * s1);
        base[j1] = from_f<T>(b * c1 - a * s0);
      }
    }
  }
}

// In-place RoPE on x[..., heads, D] (last dim contiguous). positions: optional int64 [T].
void rope_(at::Tensor& x, const c10::optional<at::Tensor>& positions, int64_t off, int64_t R, int64_t seq_len,
           double theta, int64_t mode, bool inverse) {
  TORCH_CHECK(x.stride(-1) == 1, "rope_: last dim must be contiguous");
  TORCH_CHECK(R % 2 == 0 && off + R <= x.size(-1), "rope_: bad rotary range");
  const int heads = static_cast<int>(x.size(-2));
  const int64_t sh = x.stride(-2);
  const int64_t sx = x.stride(-3);
  const int64_t T_ = x.numel() / (x.size(-1) * heads);
  TORCH_CHECK(x.dim() == 3 || x.is_contiguous() || x.stride(0) == x.size(1) * sx, "rope_: unsupported layout");
  if (T_ == 0) return;
  const int64_t total = T_ * heads * (R / 2);
  const int threads = 256;
  const int blocks = static_cast<int>(std::min<int64_t>((total + threads - 1) / threads, 148 * 16));
  auto stream = at::cuda::getCurrentCUDAStream();
  NTB_DISPATCH_FLOAT(x.scalar_type(), "rope_", [&] {
    rope_kernel<scalar_t><<<blocks, threads, 0, stream>>>(
        P<scalar_t>(x), positions.has_value() ? positions->data_ptr<int64_t>() : nullptr,
        static_cast<int>(T_), heads, sx, sh, static_cast<int>(off), static_cast<int>(R), static_cast<int>(seq_len),
        static_cast<float>(theta), static_cast<int>(mode), inverse);
  });
  NTB_LAUNCH_CHECK(1);
}

// Table-driven, vectorised RoPE for rows of a fused projection. cs[pos * (R/2) + k] = (cos, sin) of
// pos * theta^(-2k/R), built once per (seq_len, R, theta) on the host side of the binding's caller;
// positions are t % seq_len. Each thread rotates one 16-byte chunk (8 elements) in place: for the
// half-split layout the chunk of columns [i0, i0+8) together with its partner chunk [i0+R/2, ...),
// for the interleaved layout 4 adjacent (2i, 2i+1) pairs. x is [T, heads, D] with the rotary part
// at columns [off, off + R); every address involved is 16-byte aligned (checked by the binding).
template <typename T, int MODE>
__global__ void __launch_bounds__(256) rope_table_kernel(T* __restrict__ x, const float2* __restrict__ cs,
                                                         int64_t T_, int heads, int64_t sx, int64_t sh, int off,
                                                         int R, int seq_len, bool inverse) {
  const int half = R / 2;
  const int chunks = (MODE == 0 ? half : R) / 8;
  const int64_t total = T_ * heads * chunks;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % chunks);
    const int64_t th = idx / chunks;
    const int hd = static_cast<int>(th % heads);
    const int64_t t = th / heads;
    const float2* row = cs + static_cast<int64_t>(t % seq_len) * half;
    T* base = x + t * sx + hd * sh + off;
    const float sgn = inverse ? -1.f : 1.f;
    if (MODE == 0) {
      const int i0 = c * 8;
      float a[8], b[8], oa[8], ob[8];
      ld8(base + i0, a);
      ld8(base + i0 + half, b);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 q = row[i0 + j];
        const float sn = sgn * q.y;
        oa[j] = a[j] * q.x - b[j] * sn;
        ob[j] = b[j] * q.x + a[j] * sn;
      }
      st8(base + i0, oa);
      st8(base + i0 + half, ob);
    } else {
      const int j0 = c * 8;
      float v[8], o[8];
      ld8(base + j0, v);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float2 q0 = row[(j0 + 2 * m) % half], q1 = row[(j0 + 2 * m + 1) % half];
        const float a = v[2 * m], b = v[2 * m + 1];
        if (!inverse) {
          o[2 * m] = a * q0.x - b * q0.y;
          o[2 * m + 1] = b * q1.x + a * q1.y;
        } else {
          o[2 * m] = a * q0.x + b * q1.y;
          o[2 * m + 1] = b * q1.x - a * q0.y;
        }
      }
      st8(base + j0, o);
    }
  }
}

// In-place RoPE on x[T, heads, D] (last dim contiguous) from a (cos, sin) table [seq_len, R/2, 2] fp32.
void rope_table_(at::Tensor& x, const at::Tensor& table, int64_t off, int64_t R, int64_t seq_len, int64_t mode,
                 bool inverse) {
  TORCH_CHECK(x.dim() == 3 && x.stride(-1) == 1, "rope_table_: x must be [T, heads, D] with contiguous D");
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kFloat && table.is_contiguous() &&
                  table.numel() == seq_len * R,
              "rope_table_: table must be contiguous fp32 [seq_len, R/2, 2]");
  TORCH_CHECK(R % 16 == 0 && off % 8 == 0 && off + R <= x.size(-1), "rope_table_: rotary range");
  const int64_t sx = x.stride(0), sh = x.stride(1);
  TORCH_CHECK(sx % 8 == 0 && sh % 8 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0,
              "rope_table_: rows and heads must start on 16-byte boundaries");
  const int64_t T_ = x.size(0);
  const int heads = static_cast<int>(x.size(1));
  if (T_ == 0 || heads == 0) return;
  const int64_t total = T_ * heads * (mode == 0 ? R / 2 : R) / 8;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 16L * num_sms(x.get_device())));
  auto stream = at::cuda::getCurrentCUDAStream();
  const float2* cs = reinterpret_cast<const float2*>(table.data_ptr<float>());
  NTB_DISPATCH_FLOAT(x.scalar_type(), "rope_table_", [&] {
    if (mode == 0)
      rope_table_kernel<scalar_t, 0><<<blocks, 256, 0, stream>>>(P<scalar_t>(x), cs, T_, heads, sx, sh,
                                                                 static_cast<int>(off), static_cast<int>(R),
                                                                 static_cast<int>(seq_len), inverse);
    else
      rope_table_kernel<scalar_t, 1><<<blocks, 256, 0, stream>>>(P<scalar_t>(x), cs, T_, heads, sx, sh,
                                                                 static_cast<int>(off), static_cast<int>(R),
                                                                 static_cast<int>(seq_len), inverse);
  });
  NTB_LAUNCH_CHECK(1);
}

// Key assembly of multi-head latent attention. Each head's key is [nope | rope]: the nope part is
// columns [0, Dn) of that head's slice of the kv up-projection, the rope part one rotated vector per
// token that every head shares. One launch writes kf[t, h, :] = [kv[t, h, 0:Dn] | rope(kr[t, :])] in
// 16-byte chunks (interleaved-pair rotation from the (cos, sin) table, positions t % seq_len); it
// stands for a rotation launch, the broadcast over heads and the concatenation.
__global__ void __launch_bounds__(256) mla_k_assemble_kernel(const bf16* __restrict__ kv, int64_t kv_st,
                                                             int64_t kv_sh, const bf16* __restrict__ kr,
                                                             int64_t kr_st, const float2* __restrict__ cs,
                                                             bf16* __restrict__ kf, int64_t T_, int heads, int Dn,
                                                             int R, int seq_len) {
  const int cn = Dn / 8, chunks = cn + R / 8, half = R / 2;
  const int64_t total = T_ * heads * chunks;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % chunks);
    const int64_t th = idx / chunks;
    const int hd = static_cast<int>(th % heads);
    const int64_t t = th / heads;
    bf16* dst = kf + th * (Dn + R) + c * 8;
    if (c < cn) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(kv + t * kv_st + hd * kv_sh + c * 8);
      continue;
    }
    const int j0 = (c - cn) * 8;
    const float2* row = cs + static_cast<int64_t>(t % seq_len) * half;
    float v[8], o[8];
    ld8(kr + t * kr_st + j0, v);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float2 q0 = row[(j0 + 2 * m) % half], q1 = row[(j0 + 2 * m + 1) % half];
      o[2 * m] = v[2 * m] * q0.x - v[2 * m + 1] * q0.y;
      o[2 * m + 1] = v[2 * m + 1] * q1.x + v[2 * m] * q1.y;
    }
    st8(dst, o);
  }
}

// Backward of the key assembly: dkv[t, h, 0:Dn] = dk[t, h, 0:Dn] for every head, and
// dkr[t, :] = rope^T(sum over heads of dk[t, h, Dn:Dn+R]) with the head sum in fp32 and one rounding.
// One warp per token: the lanes copy the nope chunks, then lane l adds rope chunk l % (R/8) of heads
// l / (R/8), l / (R/8) + 32 / (R/8), ...; lanes holding the same chunk combine by xor shuffles (R/8
// divides 32, checked by the binding), and lanes 0 .. R/8-1 rotate back and store.
__global__ void __launch_bounds__(256) mla_k_assemble_bwd_kernel(const bf16* __restrict__ dk, int64_t dk_st,
                                                                 int64_t dk_sh, bf16* __restrict__ dkv,
                                                                 int64_t dkv_st, int64_t dkv_sh,
                                                                 bf16* __restrict__ dkr, int64_t dkr_st,
                                                                 const float2* __restrict__ cs, int64_t T_,
                                                                 int heads, int Dn, int R, int seq_len) {
  const int lane = threadIdx.x & 31;
  const int cn = Dn / 8, cr = R / 8, half = R / 2;
  const int64_t wpb = blockDim.x / 32;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * wpb;
  for (int64_t t = blockIdx.x * wpb + threadIdx.x / 32; t < T_; t += nwarps) {
    const bf16* src = dk + t * dk_st;
    bf16* dst = dkv + t * dkv_st;
    for (int i = lane; i < heads * cn; i += 32) {
      const int hd = i / cn, c = i - hd * cn;
      *reinterpret_cast<uint4*>(dst + hd * dkv_sh + c * 8) =
          *reinterpret_cast<const uint4*>(src + hd * dk_sh + c * 8);
    }
    const int rc = lane % cr;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int hd = lane / cr; hd < heads; hd += 32 / cr) {
      float v[8];
      ld8(src + hd * dk_sh + Dn + rc * 8, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
    for (int off = cr; off < 32; off <<= 1) {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], off);
    }
    if (lane < cr) {
      const int j0 = lane * 8;
      const float2* row = cs + static_cast<int64_t>(t % seq_len) * half;
      float o[8];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float2 q0 = row[(j0 + 2 * m) % half], q1 = row[(j0 + 2 * m + 1) % half];
        o[2 * m] = acc[2 * m] * q0.x + acc[2 * m + 1] * q1.y;
        o[2 * m + 1] = acc[2 * m + 1] * q1.x - acc[2 * m] * q0.y;
      }
      st8(dkr + t * dkr_st + j0, o);
    }
  }
}

static void check_mla_rows(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.stride(-1) == 1, what, ": bf16 CUDA, last dim contiguous");
  for (int d = 0; d + 1 < t.dim(); ++d) TORCH_CHECK(t.stride(d) % 8 == 0, what, ": strides must be 16-byte multiples");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, what, ": 16-byte aligned start");
}

static void check_mla_table(const at::Tensor& table, int64_t seq_len, int64_t R) {
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kFloat && table.is_contiguous() &&
                  table.numel() == seq_len * R,
              "mla_k_assemble: table must be contiguous fp32 [seq_len, R/2, 2]");
  TORCH_CHECK(R % 8 == 0 && R > 0 && 32 % (R / 8) == 0, "mla_k_assemble: R / 8 must divide 32");
}

// kv [T, heads, >= Dn], kr [T, R] -> kf [T, heads, Dn + R] (contiguous).
at::Tensor mla_k_assemble(const at::Tensor& kv, const at::Tensor& kr, const at::Tensor& table, int64_t Dn,
                          int64_t seq_len) {
  TORCH_CHECK(kv.dim() == 3 && kr.dim() == 2 && kv.size(0) == kr.size(0), "mla_k_assemble: kv [T, heads, D], kr [T, R]");
  check_mla_rows(kv, "mla_k_assemble kv");
  check_mla_rows(kr, "mla_k_assemble kr");
  const int64_t R = kr.size(1), T_ = kv.size(0), heads = kv.size(1);
  TORCH_CHECK(Dn % 8 == 0 && Dn > 0 && Dn <= kv.size(2), "mla_k_assemble: Dn");
  check_mla_table(table, seq_len, R);
  auto kf = at::empty({T_, heads, Dn + R}, kv.options());
  if (T_ == 0 || heads == 0) return kf;
  const int64_t total = T_ * heads * (Dn + R) / 8;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 16L * num_sms(kv.get_device())));
  mla_k_assemble_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      P<bf16>(kv), kv.stride(0), kv.stride(1), P<bf16>(kr), kr.stride(0),
      reinterpret_cast<const float2*>(table.data_ptr<float>()), P<bf16>(kf), T_, static_cast<int>(heads),
      static_cast<int>(Dn), static_cast<int>(R), static_cast<int>(seq_len));
  NTB_LAUNCH_CHECK(1);
  return kf;
}

// dk [T, heads, Dn + R]; writes dkv[:, :, 0:Dn] and returns dkr [T, R].
at::Tensor mla_k_assemble_bwd(const at::Tensor& dk, at::Tensor& dkv, const at::Tensor& table, int64_t Dn,
                              int64_t seq_len) {
  TORCH_CHECK(dk.dim() == 3 && dkv.dim() == 3 && dk.size(0) == dkv.size(0) && dk.size(1) == dkv.size(1),
              "mla_k_assemble_bwd: dk [T, heads, Dn + R], dkv [T, heads, >= Dn]");
  check_mla_rows(dk, "mla_k_assemble_bwd dk");
  check_mla_rows(dkv, "mla_k_assemble_bwd dkv");
  const int64_t R = dk.size(2) - Dn, T_ = dk.size(0), heads = dk.size(1);
  TORCH_CHECK(Dn % 8 == 0 && Dn > 0 && Dn <= dkv.size(2), "mla_k_assemble_bwd: Dn");
  check_mla_table(table, seq_len, R);
  auto dkr = at::empty({T_, R}, dk.options());
  if (T_ == 0) return dkr;
  if (heads == 0) return dkr.zero_();
  const int blocks = static_cast<int>(std::min<int64_t>((T_ + 7) / 8, 16L * num_sms(dk.get_device())));
  mla_k_assemble_bwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      P<bf16>(dk), dk.stride(0), dk.stride(1), P<bf16>(dkv), dkv.stride(0), dkv.stride(1), P<bf16>(dkr), dkr.stride(0),
      reinterpret_cast<const float2*>(table.data_ptr<float>()), T_, static_cast<int>(heads), static_cast<int>(Dn),
      static_cast<int>(R), static_cast<int>(seq_len));
  NTB_LAUNCH_CHECK(1);
  return dkr;
}

// =========================================================== activations
// SwiGLU over a packed [rows, 2I] tensor: gate = cols [0, I), up = cols [I, 2I).
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t rows, int I) {
  const int64_t total = rows * I;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / I;
    const int c = idx % I;
    const float g = to_f(gu[r * 2 * I + c]), u = to_f(gu[r * 2 * I + I + c]);
    const float sg = g / (1.f + __expf(-g));
    out[idx] = from_f<T>(sg * u);
  }
}

// IDX: the index type (uint32_t when rows * I < 2^31: the row / column split is then a 32-bit
// division per 8 elements instead of a 64-bit one). silu(g) = g * (1 / (1 + e^-g)) with the correctly
// rounded reciprocal.
template <typename T, typename IDX>
__global__ void swiglu_fwd_vec_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t rows, int I) {
  const IDX total = static_cast<IDX>(rows * I / 8);
  for (IDX idx = blockIdx.x * static_cast<IDX>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<IDX>(gridDim.x) * blockDim.x) {
    const IDX e = idx * 8;
    const IDX r = e / static_cast<IDX>(I);
    const IDX c = e - r * static_cast<IDX>(I);
    float g[8], u[8], o[8];
    ld8(gu + static_cast<int64_t>(r) * 2 * I + c, g);
    ld8(gu + static_cast<int64_t>(r) * 2 * I + I + c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = g[j] * __frcp_rn(1.f + __expf(-g[j])) * u[j];
    st8(out + static_cast<int64_t>(e), o);
  }
}

template <typename T, typename IDX>
__global__ void swiglu_bwd_vec_kernel(const T* __restrict__ dout, const T* __restrict__ gu, T* __restrict__ dgu,
                                      int64_t rows, int I) {
  const IDX total = static_cast<IDX>(rows * I / 8);
  for (IDX idx = blockIdx.x * static_cast<IDX>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<IDX>(gridDim.x) * blockDim.x) {
    const int64_t e = static_cast<int64_t>(idx) * 8;
    const IDX rr = static_cast<IDX>(idx * 8) / static_cast<IDX>(I);
    const int64_t r = rr;
    const int c = static_cast<int>(static_cast<IDX>(idx * 8) - rr * static_cast<IDX>(I));
    float g[8], u[8], d[8], dg[8], du[8];
    ld8(gu + r * 2 * I + c, g);
    ld8(gu + r * 2 * I + I + c, u);
    ld8(dout + e, d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float s = __frcp_rn(1.f + __expf(-g[j]));
      const float sg = g[j] * s;
      du[j] = d[j] * sg;
      dg[j] = d[j] * u[j] * (s + sg * (1.f - s));
    }
    st8(dgu + r * 2 * I + c, dg);
    st8(dgu + r * 2 * I + I + c, du);
  }
}

template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ dout, const T* __restrict__ gu, T* __restrict__ dgu,
                                  int64_t rows, int I) {
  const int64_t total = rows * I;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / I;
    const int c = idx % I;
    const float g = to_f(gu[r * 2 * I + c]), u = to_f(gu[r * 2 * I + I + c]);
    const float d = to_f(dout[idx]);
    const float s = 1.f / (1.f + __expf(-g));
    const float sg = g * s;
    dgu[r * 2 * I + I + c] = from_f<T>(d * sg);
    dgu[r * 2 * I + c] = from_f<T>(d * u * (s + sg * (1.f - s)));
  }
}

static int ew_blocks(int64_t n) { return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 32))); }

at::Tensor swiglu_fwd(const at::Tensor& gu) {
  TORCH_CHECK(gu.is_contiguous() && gu.size(-1) % 2 == 0, "swiglu_fwd: packed [.., 2I] contiguous");
  const int I = static_cast<int>(gu.size(-1) / 2);
  const int64_t rows = gu.numel() / (2 * I);
  auto sizes = gu.sizes().vec();
  sizes.back() = I;
  auto out = at::empty(sizes, gu.options());
  if (rows == 0) return out;
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool vec = I % 8 == 0;
  NTB_DISPATCH_FLOAT(gu.scalar_type(), "swiglu_fwd", [&] {
    if (vec)
      if (rows * I < (1LL << 31))
        swiglu_fwd_vec_kernel<scalar_t, uint32_t><<<ew_blocks(rows * I / 8), 256, 0, stream>>>(P<scalar_t>(gu),
                                                                                             P<scalar_t>(out), rows, I);
      else
        swiglu_fwd_vec_kernel<scalar_t, int64_t><<<ew_blocks(rows * I / 8), 256, 0, stream>>>(P<scalar_t>(gu),
                                                                                            P<scalar_t>(out), rows, I);
    else
      swiglu_fwd_kernel<scalar_t><<<ew_blocks(rows * I), 256, 0, stream>>>(P<scalar_t>(gu), P<scalar_t>(out), rows, I);
  });
  NTB_LAUNCH_CHECK(1);
  return out;
}

at::Tensor swiglu_bwd(const at::Tensor& dout, const at::Tensor& gu) {
  const int I = static_cast<int>(gu.size(-1) / 2);
  const int64_t rows = gu.numel() / (2 * I);
  auto dgu = at::empty_like(gu);
  if (rows == 0) return dgu;
  auto d = dout.contiguous();
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool vec = I % 8 == 0;
  NTB_DISPATCH_FLOAT(gu.scalar_type(), "swiglu_bwd", [&] {
    if (vec)
      if (rows * I < (1LL << 31))
        swiglu_bwd_vec_kernel<scalar_t, uint32_t><<<ew_blocks(rows * I / 8), 256, 0, stream>>>(
            P<scalar_t>(d), P<scalar_t>(gu), P<scalar_t>(dgu), rows, I);
      else
        swiglu_bwd_vec_kernel<scalar_t, int64_t><<<ew_blocks(rows * I / 8), 256, 0, stream>>>(
            P<scalar_t>(d), P<scalar_t>(gu), P<scalar_t>(dgu), rows, I);
    else
      swiglu_bwd_kernel<scalar_t><<<ew_blocks(rows * I), 256, 0, stream>>>(P<scalar_t>(d), P<scalar_t>(gu),
                                                                          P<scalar_t>(dgu), rows, I);
  });
  NTB_LAUNCH_CHECK(1);
  return dgu;
}

// Exact GELU x * Phi(x) using CUDA's erff.
template <typename T>
__global__ void gelu_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = to_f(x[i]);
    y[i] = from_f<T>(0.5f * v * (1.f + erff(v * 0.70710678118654752f)));
  }
}
template <typename T>
__global__ void gelu_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x, T* __restrict__ dx, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = to_f(x[i]);
    const float cdf = 0.5f * (1.f + erff(v * 0.70710678118654752f));
    const float pdf = 0.3989422804014327f * __expf(-0.5f * v * v);
    dx[i] = from_f<T>(to_f(dy[i]) * (cdf + v * pdf));
  }
}

at::Tensor gelu_fwd(const at::Tensor& x) {
  auto xc = x.contiguous();
  auto y = at::empty_like(xc);
  const int64_t n = xc.numel();
  if (n == 0) return y;
  auto stream = at::cuda::getCurrentCUDAStream();
  NTB_DISPATCH_FLOAT(x.scalar_type(), "gelu_fwd", [&] {
    gelu_fwd_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream>>>(P<scalar_t>(xc), P<scalar_t>(y), n);
  });
  NTB_LAUNCH_CHECK(1);
  return y;
}

at::Tensor gelu_bwd(const at::Tensor& dy, const at::Tensor& x) {
  auto xc = x.contiguous();
  auto d = dy.contiguous();
  auto dx = at::empty_like(xc);
  const int64_t n = xc.numel();
  if (n == 0) return dx;
  auto stream = at::cuda::getCurrentCUDAStream();
  NTB_DISPATCH_FLOAT(x.scalar_type(), "gelu_bwd", [&] {
    gelu_bwd_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream>>>(P<scalar_t>(d), P<scalar_t>(xc),
                                                              P<scalar_t>(dx), n);
  });
  NTB_LAUNCH_CHECK(1);
  return dx;
}

// =========================================================== cross-entropy
// Per-row statistics of a (possibly vocab-sharded) logits block [rows, V]:
//   row_max, row_sumexp (relative to row_max), target logit (0 if the label
//   is outside [vstart, vstart + V) or equals ignore_index).
template <typename T>
__global__ void ce_stats_kernel(const T* __restrict__ logits, int64_t ld, const int64_t* __restrict__ labels,
                                int64_t V, int64_t vstart, int64_t ignore_index, float* __restrict__ out_max,
                                float* __restrict__ out_sum, float* __restrict__ out_tgt) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* lr = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  const bool vec = (V % 8 == 0) && (ld % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  if (vec) {
    for (int64_t i = threadIdx.x * 8; i < V; i += blockDim.x * 8) {
      float v[8];
      ld8(lr + i, v);
      float lm = v[0];
#pragma unroll
      for (int j = 1; j < 8; ++j) lm = fmaxf(lm, v[j]);
      const float nm = fmaxf(m, lm);
      float acc = s * __expf(m - nm);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc += __expf(v[j] - nm);
      s = acc;
      m = nm;
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
      const float v = to_f(lr[i]);
      const float nm = fmaxf(m, v);
      s = s * __expf(m - nm) + __expf(v - nm);
      m = nm;
    }
  }
  const float gm = block_max(m, red);
  float sc = (m == -INFINITY) ? 0.f : s * __expf(m - gm);
  sc = block_sum(sc, red);
  if (threadIdx.x == 0) {
    out_max[row] = gm;
    out_sum[row] = sc;
    const int64_t lab = labels[row];
    float t = 0.f;
    if (lab != ignore_index && lab >= vstart && lab < vstart + V) t = to_f(lr[lab - vstart]);
    out_tgt[row] = t;
  }
}

// grad[row, j] = (exp(x - lse[row]) - [j + vstart == label]) * scale[row or 0], 0 for ignored rows.
template <typename T, typename G>
__global__ void ce_bwd_kernel(const T* __restrict__ logits, int64_t ld, const int64_t* __restrict__ labels,
                              const float* __restrict__ lse, const float* __restrict__ scale, int scale_per_row,
                              int64_t V, int64_t vstart, int64_t ignore_index, G* __restrict__ grad, int64_t ldg) {
  const int64_t row = blockIdx.x;
  const int64_t lab = labels[row];
  const T* lr = logits + row * ld;
  G* gr = grad + row * ldg;
  const float sc = scale[scale_per_row ? row : 0];
  const float l = lse[row];
  const bool ign = (lab == ignore_index);
  const bool vec = (V % 8 == 0) && (ld % 8 == 0) && (ldg % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(logits) & 15) == 0) && ((reinterpret_cast<uintptr_t>(grad) & 15) == 0);
  if (vec) {
    for (int64_t i = threadIdx.x * 8; i < V; i += blockDim.x * 8) {
      float v[8];
      ld8(lr + i, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float g = ign ? 0.f : __expf(v[j] - l);
        if (!ign && i + j + vstart == lab) g -= 1.f;
        v[j] = g * sc;
      }
      st8(gr + i, v);
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
      float g = ign ? 0.f : __expf(to_f(lr[i]) - l);
      if (!ign && i + vstart == lab) g -= 1.f;
      gr[i] = from_f<G>(g * sc);
    }
  }
}

std::vector<at::Tensor> ce_stats(const at::Tensor& logits, const at::Tensor& labels, int64_t vstart,
                                 int64_t ignore_index) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "ce_stats: 2-D logits with unit inner stride");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous(), "ce_stats: int64 labels");
  const int64_t rows = logits.size(0), V = logits.size(1);
  auto opts = logits.options().dtype(at::kFloat);
  auto mx = at::empty({rows}, opts), sm = at::empty({rows}, opts), tg = at::empty({rows}, opts);
  if (rows == 0) return {mx, sm, tg};
  auto stream = at::cuda::getCurrentCUDAStream();
  NTB_DISPATCH_FLOAT(logits.scalar_type(), "ce_stats", [&] {
    ce_stats_kernel<scalar_t><<<rows, 1024, 0, stream>>>(P<scalar_t>(logits), logits.stride(0),
                                                         labels.data_ptr<int64_t>(), V, vstart, ignore_index,
                                                         mx.data_ptr<float>(), sm.data_ptr<float>(), tg.data_ptr<float>());
  });
  NTB_LAUNCH_CHECK(1);
  return {mx, sm, tg};
}

// Writes the CE gradient into `grad` (may alias `logits`).
void ce_bwd(const at::Tensor& logits, const at::Tensor& labels, const at::Tensor& lse, const at::Tensor& scale,
            int64_t vstart, int64_t ignore_index, at::Tensor& grad) {
  const int64_t rows = logits.size(0), V = logits.size(1);
  if (rows == 0) return;
  TORCH_CHECK(scale.scalar_type() == at::kFloat && (scale.numel() == 1 || scale.numel() == rows), "ce_bwd: scale");
  TORCH_CHECK(grad.scalar_type() == logits.scalar_type() && grad.stride(1) == 1, "ce_bwd: grad");
  auto stream = at::cuda::getCurrentCUDAStream();
  NTB_DISPATCH_FLOAT(logits.scalar_type(), "ce_bwd", [&] {
    ce_bwd_kernel<scalar_t, scalar_t><<<rows, 1024, 0, stream>>>(
        P<scalar_t>(logits), logits.stride(0), labels.data_ptr<int64_t>(), lse.data_ptr<float>(),
        scale.data_ptr<float>(), scale.numel() == rows ? 1 : 0, V, vstart, ignore_index, P<scalar_t>(grad),
        grad.stride(0));
  });
  NTB_LAUNCH_CHECK(1);
}

// =========================================================== embedding
template <typename T>
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const T* __restrict__ W, T* __restrict__ out,
                                     int64_t n, int H, int64_t vstart, int64_t vcount, int* status) {
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t] - vstart;
  T* o = out + t * H;
  if (id < 0 || id >= vcount) {
    // Outside this shard (vocab-parallel) -> zeros.
    for (int i = threadIdx.x; i < H; i += blockDim.x) o[i] = from_f<T>(0.f);
    return;
  }
  const T* w = W + id * H;
  if ((H % 8 == 0) && sizeof(T) == 2) {
    for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8)
      *reinterpret_cast<uint4*>(o + i) = *reinterpret_cast<const uint4*>(w + i);
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) o[i] = w[i];
  }
}

template <typename T>
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids, const T* __restrict__ dout,
                                     float* __restrict__ dW, int64_t n, int H, int64_t vstart, int64_t vcount) {
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t] - vstart;
  if (id < 0 || id >= vcount) return;
  const T* d = dout + t * H;
  float* g = dW + id * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) atomicAdd(g + i, to_f(d[i]));
}

at::Tensor embedding_fwd(const at::Tensor& ids, const at::Tensor& W, int64_t vstart) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && W.is_contiguous(), "embedding_fwd: int64 ids, contiguous weight");
  auto idc = ids.contiguous();
  const int64_t n = idc.numel(), H = W.size(1);
  auto sizes = ids.sizes().vec();
  sizes.push_back(H);
  auto out = at::empty(sizes, W.options());
  if (n == 0) return out;
  auto stream = at::cuda::getCurrentCUDAStream();
  NTB_DISPATCH_FLOAT(W.scalar_type(), "embedding_fwd", [&] {
    embedding_fwd_kernel<scalar_t><<<n, 128, 0, stream>>>(idc.data_ptr<int64_t>(), P<scalar_t>(W),
                                                          P<scalar_t>(out), n, H, vstart, W.size(0), nullptr);
  });
  NTB_LAUNCH_CHECK(1);
  return out;
}

// Accumulates the embedding gradient into an fp32 buffer dW [V, H].
void embedding_bwd_(const at::Tensor& ids, const at::Tensor& dout, at::Tensor& dW, int64_t vstart) {
  TORCH_CHECK(dW.scalar_type() == at::kFloat && dW.is_contiguous(), "embedding_bwd_: fp32 contiguous dW");
  auto idc = ids.contiguous();
  auto d = dout.contiguous();
  const int64_t n = idc.numel(), H = dW.size(1);
  if (n == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  NTB_DISPATCH_FLOAT(d.scalar_type(), "embedding_bwd_", [&] {
    embedding_bwd_kernel<scalar_t><<<n, 256, 0, stream>>>(idc.data_ptr<int64_t>(), P<scalar_t>(d),
                                                          dW.data_ptr<float>(), n, H, vstart, dW.size(0));
  });
  NTB_LAUNCH_CHECK(1);
}

// =========================================================== AdamW (flat)
// torch.optim.AdamW semantics on flat fp32 state:
//   p *= 1 - lr*wd ; m = b1 m + (1-b1) g ; v = b2 v + (1-b2) g^2
//   p -= (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps)
// grad is read as fp32 or bf16 and multiplied by grad_scale[0] (unscale /
// averaging folded in); an optional bf16 copy of the new parameter is written.
template <typename G>
__global__ void adamw_kernel(float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
                             const G* __restrict__ g, bf16* __restrict__ p_bf16, int64_t n, float lr, float b1,
                             float b2, float eps, float wd, float bc1, float sqrt_bc2,
                             const float* __restrict__ grad_scale, const int* __restrict__ skip) {
  if (skip && *skip) return;
  const float gs = grad_scale ? *grad_scale : 1.f;
  const float step = lr / bc1;
  const float decay = 1.f - lr * wd;
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float gg[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) gg[j] = to_f(g[i * 4 + j]) * gs;
    float* P = &pp.x;
    float* M = &mm.x;
    float* Vv = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      P[j] *= decay;
      M[j] = b1 * M[j] + (1.f - b1) * gg[j];
      Vv[j] = b2 * Vv[j] + (1.f - b2) * gg[j] * gg[j];
      P[j] -= step * M[j] / (sqrtf(Vv[j]) / sqrt_bc2 + eps);
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (p_bf16) {
      uint2 o;
      o.x = pack_bf16x2(pp.x, pp.y);
      o.y = pack_bf16x2(pp.z, pp.w);
      reinterpret_cast<uint2*>(p_bf16)[i] = o;
    }
  }
  for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gg = to_f(g[i]) * gs;
    float pp = p[i] * decay;
    const float mm = b1 * m[i] + (1.f - b1) * gg;
    const float vv = b2 * v[i] + (1.f - b2) * gg * gg;
    pp -= step * mm / (sqrtf(vv) / sqrt_bc2 + eps);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
    if (p_bf16) p_bf16[i] = __float2bfloat16(pp);
  }
}

void adamw_flat_(at::Tensor& p, at::Tensor& m, at::Tensor& v, const at::Tensor& g,
                 const c10::optional<at::Tensor>& p_bf16, double lr, double b1, double b2, double eps, double wd,
                 int64_t step, const c10::optional<at::Tensor>& grad_scale, const c10::optional<at::Tensor>& skip) {
  TORCH_CHECK(p.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat,
              "adamw_flat_: fp32 state");
  TORCH_CHECK(p.is_contiguous() && m.is_contiguous() && v.is_contiguous() && g.is_contiguous(), "adamw_flat_: contiguous");
  const int64_t n = p.numel();
  TORCH_CHECK(m.numel() == n && v.numel() == n && g.numel() == n, "adamw_flat_: sizes");
  if (p_bf16.has_value()) TORCH_CHECK(p_bf16->numel() == n && p_bf16->scalar_type() == at::kBFloat16 && p_bf16->is_contiguous(), "adamw_flat_: p_bf16");
  if (n == 0) return;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(p.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(m.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(v.data_ptr()) & 15) == 0,
              "adamw_flat_: 16B alignment");
  if (p_bf16.has_value()) TORCH_CHECK((reinterpret_cast<uintptr_t>(p_bf16->data_ptr()) & 7) == 0, "adamw_flat_: p_bf16 8B alignment");
  const float bc1 = 1.f - static_cast<float>(std::pow(b1, static_cast<double>(step)));
  const float bc2 = 1.f - static_cast<float>(std::pow(b2, static_cast<double>(step)));
  auto stream = at::cuda::getCurrentCUDAStream();
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n / 4 + 255) / 256, num_sms(p.get_device()) * 8)));
  const float* gs = grad_scale.has_value() ? grad_scale->data_ptr<float>() : nullptr;
  const int* sk = skip.has_value() ? skip->data_ptr<int>() : nullptr;
  bf16* pb = p_bf16.has_value() ? reinterpret_cast<bf16*>(p_bf16->data_ptr()) : nullptr;
  NTB_DISPATCH_FLOAT(g.scalar_type(), "adamw_flat_", [&] {
    adamw_kernel<scalar_t><<<blocks, 256, 0, stream>>>(p.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                                                       P<scalar_t>(g), pb, n, lr, b1, b2, eps, wd, bc1,
                                                       std::sqrt(bc2), gs, sk);
  });
  NTB_LAUNCH_CHECK(1);
}

// =========================================================== unscale / finite / sum of squares
// g *= inv_scale (in place, optional) ; out[0] += sum(g^2) ; out[1] = 1 if any non-finite.
template <typename T>
__global__ void grad_stats_kernel(T* __restrict__ g, int64_t n, const float* __restrict__ inv_scale,
                                  float* __restrict__ out) {
  __shared__ float red[32];
  const float s = inv_scale ? *inv_scale : 1.f;
  float ss = 0.f;
  int bad = 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v = to_f(g[i]);
    if (inv_scale) {
      v *= s;
      g[i] = from_f<T>(v);
    }
    if (!isfinite(v)) bad = 1;
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const int anybad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    atomicAdd(out, ss);
    if (anybad) out[1] = 1.f;
  }
}

// fp32 form with 16-byte accesses and two of them in flight per thread (the scalar form keeps
// too few bytes in flight to reach HBM bandwidth); the n % 4 tail is handled by block 0.
__global__ void __launch_bounds__(256) grad_stats_vec_kernel(float* __restrict__ g, int64_t n,
                                                             const float* __restrict__ inv_scale,
                                                             float* __restrict__ out) {
  __shared__ float red[32];
  const float s = inv_scale ? *inv_scale : 1.f;
  float ss = 0.f;
  int bad = 0;
  float4* g4 = reinterpret_cast<float4*>(g);
  const int64_t n4 = n / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  auto take = [&](float4& v, int64_t i) {
    if (inv_scale) {
      v.x *= s; v.y *= s; v.z *= s; v.w *= s;
      g4[i] = v;
    }
    bad |= !(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w));
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  };
  int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  for (; i + stride < n4; i += 2 * stride) {
    float4 a = g4[i], b = g4[i + stride];
    take(a, i);
    take(b, i + stride);
  }
  if (i < n4) {
    float4 a = g4[i];
    take(a, i);
  }
  if (blockIdx.x == 0 && threadIdx.x < n - n4 * 4) {
    const int64_t j = n4 * 4 + threadIdx.x;
    float v = g[j];
    if (inv_scale) {
      v *= s;
      g[j] = v;
    }
    bad |= !isfinite(v);
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const int anybad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    atomicAdd(out, ss);
    if (anybad) out[1] = 1.f;
  }
}

// Returns nothing; accumulates into out (fp32 [2]: sumsq, nonfinite flag).
void grad_stats_(at::Tensor& g, const c10::optional<at::Tensor>& inv_scale, at::Tensor& out) {
  TORCH_CHECK(g.is_contiguous() && out.scalar_type() == at::kFloat && out.numel() >= 2, "grad_stats_");
  const int64_t n = g.numel();
  if (n == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, num_sms(g.get_device()) * 4)));
  if (g.scalar_type() == at::kFloat && (reinterpret_cast<uintptr_t>(g.data_ptr()) & 15) == 0) {
    const int vblocks = static_cast<int>(
        std::max<int64_t>(1, std::min<int64_t>((n / 4 + 511) / 512, num_sms(g.get_device()) * 8)));
    grad_stats_vec_kernel<<<vblocks, 256, 0, stream>>>(g.data_ptr<float>(), n,
                                                       inv_scale.has_value() ? inv_scale->data_ptr<float>() : nullptr,
                                                       out.data_ptr<float>());
    NTB_LAUNCH_CHECK(1);
    return;
  }
  NTB_DISPATCH_FLOAT(g.scalar_type(), "grad_stats_", [&] {
    grad_stats_kernel<scalar_t><<<blocks, 256, 0, stream>>>(P<scalar_t>(g), n,
                                                            inv_scale.has_value() ? inv_scale->data_ptr<float>() : nullptr,
                                                            out.data_ptr<float>());
  });
  NTB_LAUNCH_CHECK(1);
}

}  // namespace ntb
