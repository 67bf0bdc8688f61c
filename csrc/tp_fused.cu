// Fused tensor-parallel compute + collective kernels over NVLink peer memory.
//
// ag_gemm:  Y[T, N] = AllGather_T(X_shard)[T, K] . op(W)^T        (ColumnParallel fwd,
//           also returns the gathered X for the weight gradient)   RowParallel bwd dgrad)
// gemm_rs:  Y_shard[T/n, N] = ReduceScatter_T(X[T, K] . op(W)^T)  (RowParallel fwd,
//                                                                   ColumnParallel bwd dgrad)
//
// Both are ONE cooperative launch of persistent CTAs on every rank of the
// tensor-parallel group; the GEMM core is the same tcgen05/TMA/TMEM pipeline
// as gemm.cu (128 x BN x 64 tiles, 2 TMEM accumulators, warp roles
// TMA / MMA / 4 epilogue warps).
//
// ag_gemm: CTAs [0, C) are copy CTAs. Each rank first publishes "my shard of
// this epoch is in my symmetric slot" (a release store of the epoch into its
// ready word). Copy CTAs walk the chunks in rank-rotated order (own chunk
// first), wait (bounded) for the owner's ready word, and stream their slice
// of the owner's shard into the local gathered buffer with bulk-async copies
// (cp.async.bulk peer-global -> shared -> local-global, several 32 KB pieces in
// flight, no cluster multicast). Each finished slice bumps a local per-chunk
// counter. GEMM CTAs walk their tiles in the same chunk order and the TMA
// producer waits on the chunk counter before the first A load of a chunk, so
// the tiles of chunk j run while chunk j+1 is still crossing NVLink.
//
// gemm_rs: every CTA runs GEMM tiles ordered by destination chunk (peers
// first, own chunk last). The epilogue stores each bf16 tile directly into the
// destination rank's receive slot for this source rank and then, after a
// system-scope fence, adds one to the destination's arrival counter. When a CTA
// runs out of tiles it joins the reduction of this rank's chunk: it waits
// (bounded) until all n * tiles_per_chunk tiles have arrived and sums the n
// slots (+ bias) into the output.
//
// Buffers alternate between two slots by epoch parity; a rank reuses a slot
// only two calls later, by which time every peer has finished the call that
// read it (each call waits on every peer's data of the previous epoch).
// Every wait is bounded and reports through the status word.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace ntb {

using bf16 = __nv_bfloat16;
constexpr int kMaxRanks = 8;

// ------------------------------------------------------------------ scoped memory ops
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned int ld_acquire_gpu_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys_add(unsigned int* p, unsigned int v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Bounded spin until pred() holds; records `code` and returns false on timeout.
template <typename F>
__device__ __forceinline__ bool spin_until(F pred, int* status, int code) {
  if (pred()) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (true) {
    if (pred()) return true;
    if ((++n & 63u) == 0) {
      if (status_raised(status)) return false;
      if (globaltimer_ns() - t0 > NTB_WAIT_LIMIT_NS) {
        set_status(status, code);
        return false;
      }
    }
  }
}

// Bulk-async copies (TMA engine, non-tensor form, no multicast).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_store(void* gdst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(smem_src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ------------------------------------------------------------------ shared GEMM core
template <int BN>
struct FusedCfg {
  static constexpr int BM = 128, BK = 64, STAGES = (BN == 256) ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = 1024 + STAGES * (A_BYTES + B_BYTES) + 512;
  static constexpr int COPY_PIECE = 32768;
  static constexpr int COPY_BUFS = (STAGES * (A_BYTES + B_BYTES)) / COPY_PIECE;
};

struct AgParams {
  int M, N, K;          // M = n * T_local
  int T_local, n, rank, copy_ctas;
  unsigned long long epoch;
  bf16* full;                                  // local gathered X [M, K]
  const bf16* x_local;                         // this rank's shard [T_local, K] (kernel fills the slot from it)
  bf16* my_slot;                               // this rank's symmetric slot for this epoch
  const bf16* peer_slot[kMaxRanks];            // each rank's shard slot [T_local, K] (this epoch)
  const unsigned long long* peer_ready[kMaxRanks];
  unsigned long long* my_ready;
  unsigned int* chunk_flags;                   // local [n], += copy_ctas per epoch
  unsigned int* tile_ctr;                      // local, zeroed before the launch
  bf16* C;
  long ldc;
  const bf16* bias;
  int* status;
};

struct RsParams {
  int M, N, K;          // M = n * T_local (full rows of the partial product)
  int T_local, n, rank;
  unsigned long long epoch;
  bf16* peer_recv[kMaxRanks];                  // each rank's receive slot base [n][T_local][N] (this epoch)
  unsigned int* peer_counter[kMaxRanks];       // each rank's arrival counter (this epoch parity)
  unsigned int* my_counter;
  const bf16* my_recv;
  unsigned int* tile_ctr;                      // local, zeroed before the launch
  bf16* out;                                   // [T_local, N]
  long ldo;
  const bf16* bias;
  int* status;
};

// Tile t -> (mb, nb) with chunks visited in rank-rotated order starting at
// `first_step` and M fastest inside a chunk.
__device__ __forceinline__ void rotated_tile(int t, int tiles_per_chunk, int mtiles_per_chunk, int n, int rank,
                                             int first_step, int& mb, int& nb, int& chunk) {
  const int s = t / tiles_per_chunk + first_step;
  const int r = t % tiles_per_chunk;
  chunk = (rank + s) % n;
  mb = chunk * mtiles_per_chunk + r % mtiles_per_chunk;
  nb = r / mtiles_per_chunk;
}


// ------------------------------------------------------------------ dynamic-tile GEMM phase
// Shared-memory layout of one CTA (after 1024-byte alignment):
//   [0, STAGES*A)            A ring        [STAGES*A, STAGES*(A+B))   B ring
//   barriers: full[S] empty[S] tfull[2] tempty[2] tdone[2] drain tring_full[4] tring_empty[4] copy_bars[8]
//   tile ring int[4], TMEM base slot
template <int BN>
struct FusedSmem {
  using Cfg = FusedCfg<BN>;
  uint8_t* sA;
  uint8_t* sB;
  uint64_t *full, *empty, *tfull, *tempty, *tdone, *drain, *tring_full, *tring_empty, *copy_bars;
  int* tring;
  uint32_t* tmem_slot;
  __device__ __forceinline__ explicit FusedSmem(uint8_t* smem) {
    sA = smem;
    sB = smem + Cfg::STAGES * Cfg::A_BYTES;
    full = reinterpret_cast<uint64_t*>(sB + Cfg::STAGES * Cfg::B_BYTES);
    empty = full + Cfg::STAGES;
    tfull = empty + Cfg::STAGES;
    tempty = tfull + 2;
    tdone = tempty + 2;
    drain = tdone + 2;
    tring_full = drain + 1;
    tring_empty = tring_full + 4;
    copy_bars = tring_empty + 4;
    tring = reinterpret_cast<int*>(copy_bars + 8);
    tmem_slot = reinterpret_cast<uint32_t*>(tring + 4);
  }
  __device__ __forceinline__ void init() {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
      mbar_init(&tdone[b], 128);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&tring_full[b], 1);
      mbar_init(&tring_empty[b], 128);
    }
    mbar_init(drain, 1);
    for (int b = 0; b < 8; ++b) mbar_init(&copy_bars[b], 1);
    mbar_fence_init();
  }
};

// Runs GEMM tiles handed out by a global atomic counter. `tile_of(t, mb, nb, chunk)` maps
// a tile index; `wait_chunk(chunk)` (producer) gates A loads; `store(t_row_taddr, row, mb, nb, chunk)`
// is the per-tile epilogue of one thread's TMEM row; `published(chunk)` runs once per tile after all
// epilogue threads stored (one thread).
template <int BN, bool B_MN, bool PUBLISH, typename TileOf, typename WaitChunk, typename Store, typename Published>
__device__ __forceinline__ void gemm_phase(FusedSmem<BN>& sm, uint32_t tmem_base, const CUtensorMap* tmA,
                                           const CUtensorMap* tmB, int K, int num_tiles, unsigned int* tile_ctr,
                                           int* status, TileOf tile_of, WaitChunk wait_chunk, Store store,
                                           Published published, const CUtensorMap* tmA_own = nullptr,
                                           int own_chunk = -1, int mtiles_per_chunk = 0) {
  using Cfg = FusedCfg<BN>;
  constexpr int BM = Cfg::BM, BK = Cfg::BK, STAGES = Cfg::STAGES;
  constexpr int A_BYTES = Cfg::A_BYTES, B_BYTES = Cfg::B_BYTES;
  constexpr uint32_t IDESC = make_idesc_f16(BM, BN, false, B_MN);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_kb = (K + BK - 1) / BK;
  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, filled_mask = 0;
      uint32_t last_phase[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_phase[s] = 0;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int slot = i & 3;
        const uint32_t par = static_cast<uint32_t>((i >> 2) & 1);
        if (!mbar_wait(&sm.tring_empty[slot], par ^ 1, status, kStatusTimeoutProducer)) break;
        const int t = static_cast<int>(atomicAdd(tile_ctr, 1u));
        const int tt = t < num_tiles ? t : -1;
        sm.tring[slot] = tt;
        mbar_arrive(&sm.tring_full[slot]);
        if (tt < 0) break;
        int mb, nb, chunk;
        tile_of(tt, mb, nb, chunk);
        if (!wait_chunk(chunk)) break;
        const bool own = (tmA_own != nullptr) && (chunk == own_chunk);
        const CUtensorMap* amap = own ? tmA_own : tmA;
        const int arow = own ? (mb - own_chunk * mtiles_per_chunk) * BM : mb * BM;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&sm.empty[stage], phase ^ 1, status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&sm.full[stage], A_BYTES + B_BYTES);
          tma_load_2d(sm.sA + stage * A_BYTES, amap, &sm.full[stage], kb * BK, arow);
          if constexpr (!B_MN) {
            tma_load_2d(sm.sB + stage * B_BYTES, tmB, &sm.full[stage], kb * BK, nb * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sm.sB + stage * B_BYTES + j * 8192, tmB, &sm.full[stage], nb * BN + j * 64, kb * BK);
          }
          filled_mask |= 1u << stage;
          last_phase[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (filled_mask & (1u << s)) mbar_wait(&sm.full[s], last_phase[s], nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int slot = i & 3;
        const uint32_t par = static_cast<uint32_t>((i >> 2) & 1);
        if (!mbar_wait(&sm.tring_full[slot], par, status, kStatusTimeoutMma)) break;
        if (sm.tring[slot] < 0) break;
        if (!mbar_wait(&sm.tempty[acc], acc_phase ^ 1, status, kStatusTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&sm.full[stage], phase, status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sm.sA + stage * A_BYTES), b_base = smem_u32(sm.sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = make_smem_desc_sw128(a_base + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_smem_desc_sw128(b_base + k * 2048, 8192, 1024)
                                        : make_smem_desc_sw128(b_base + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, adesc, bdesc, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&sm.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&sm.tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      umma_commit(sm.drain);
      mbar_wait(sm.drain, 0, nullptr, 0);
    }
  } else {
    const int q = warp & 3, row = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int i = 0;; ++i) {
      const int slot = i & 3;
      const uint32_t par = static_cast<uint32_t>((i >> 2) & 1);
      if (!mbar_wait(&sm.tring_full[slot], par, status, kStatusTimeoutEpilogue)) break;
      const int t = sm.tring[slot];
      if (t < 0) break;
      int mb, nb, chunk;
      tile_of(t, mb, nb, chunk);
      if (!mbar_wait(&sm.tfull[acc], acc_phase, status, kStatusTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      store(t_row, row, mb, nb, chunk);
      tc_fence_before();
      mbar_arrive(&sm.tempty[acc]);
      if constexpr (PUBLISH) {
        __threadfence_system();
        mbar_arrive(&sm.tdone[acc]);
        if (warp == 2 && lane == 0) {
          if (mbar_wait(&sm.tdone[acc], acc_phase, status, kStatusTimeoutEpilogue)) published(chunk);
        }
      }
      mbar_arrive(&sm.tring_empty[slot]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
}

// ================================================================== AG + GEMM
template <int BN, bool B_MN>
__global__ void __launch_bounds__(192, 1)
    ag_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA_local, AgParams p) {
  using Cfg = FusedCfg<BN>;
  constexpr int BM = Cfg::BM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  FusedSmem<BN> sm(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) sm.init();
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmA_local);
  }
  if (warp == 1) {
    tmem_alloc(sm.tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *sm.tmem_slot;

  // ------------------------------------------------------------ copy phase (first C CTAs)
  if (static_cast<int>(blockIdx.x) < p.copy_ctas && threadIdx.x == 0) {
    uint64_t* bars = sm.copy_bars;
    const int c = blockIdx.x, C = p.copy_ctas;
    const int64_t chunk_bytes = static_cast<int64_t>(p.K) * 2 * p.T_local;
    const int64_t per = ((chunk_bytes / C) + 15) / 16 * 16;
    const int64_t lo = min(chunk_bytes, per * c), hi = min(chunk_bytes, per * (c + 1));
    const int64_t pieces_per_chunk = (hi - lo + Cfg::COPY_PIECE - 1) / Cfg::COPY_PIECE;
    const int64_t total = pieces_per_chunk * p.n;
    bool ok = true;
    int waited_mask = 0;
    uint32_t pending = 0, pend_parity = 0;
    auto piece = [&](int64_t i, int64_t& off, uint32_t& bytes, int& j) -> const uint8_t* {
      const int s = static_cast<int>(i / pieces_per_chunk);
      j = (p.rank + s) % p.n;
      off = lo + (i % pieces_per_chunk) * Cfg::COPY_PIECE;
      bytes = static_cast<uint32_t>(min(static_cast<int64_t>(Cfg::COPY_PIECE), hi - off));
      // Step 0 reads this rank's own shard from local memory; later steps read peer slots.
      return (s == 0 ? reinterpret_cast<const uint8_t*>(p.x_local) : reinterpret_cast<const uint8_t*>(p.peer_slot[j])) +
             off;
    };
    auto ensure_ready = [&](int j) -> bool {
      if (j == p.rank) return true;  // own shard: local source
      if (waited_mask & (1 << j)) return true;
      const unsigned long long* rw = p.peer_ready[j];
      const unsigned long long want = p.epoch;
      if (!spin_until([&] { return ld_acquire_sys_u64(rw) >= want; }, p.status, kStatusTimeoutPeer)) return false;
      waited_mask |= 1 << j;
      return true;
    };
    auto issue = [&](int64_t i) -> bool {
      int64_t off;
      uint32_t bytes;
      int j;
      const uint8_t* src = piece(i, off, bytes, j);
      if (!ensure_ready(j)) return false;
      const int b = static_cast<int>(i % Cfg::COPY_BUFS);
      mbar_expect_tx(&bars[b], bytes);
      bulk_load(smem + b * Cfg::COPY_PIECE, src, bytes, &bars[b]);
      pending |= 1u << b;
      pend_parity = (pend_parity & ~(1u << b)) | (static_cast<uint32_t>((i / Cfg::COPY_BUFS) & 1) << b);
      return true;
    };
    for (int64_t i = 0; i < min(total, static_cast<int64_t>(Cfg::COPY_BUFS)) && ok; ++i) ok = issue(i);
    int64_t done_in_chunk = 0;
    for (int64_t i = 0; i < total && ok; ++i) {
      const int b = static_cast<int>(i % Cfg::COPY_BUFS);
      if (!mbar_wait(&bars[b], static_cast<uint32_t>((i / Cfg::COPY_BUFS) & 1), p.status, kStatusTimeoutPeer)) {
        ok = false;
        break;
      }
      pending &= ~(1u << b);
      int64_t off;
      uint32_t bytes;
      int j;
      piece(i, off, bytes, j);
      bulk_store(reinterpret_cast<uint8_t*>(p.full + static_cast<int64_t>(j) * p.T_local * p.K) + off,
                 smem + b * Cfg::COPY_PIECE, bytes);
      if (j == p.rank) bulk_store(reinterpret_cast<uint8_t*>(p.my_slot) + off, smem + b * Cfg::COPY_PIECE, bytes);
      bulk_commit();
      if (++done_in_chunk == pieces_per_chunk) {
        bulk_wait_all();
        fence_proxy_async_global();
        if (j == p.rank) {
          // Own shard is in the symmetric slot: the copy CTA that completes it publishes the epoch to peers.
          __threadfence_system();
          const unsigned int prev = atomicAdd(&p.chunk_flags[j], 1u);
          if (prev + 1u == static_cast<unsigned int>(p.epoch) * static_cast<unsigned int>(p.copy_ctas))
            st_release_sys_u64(p.my_ready, p.epoch);
        } else {
          __threadfence();
          red_release_gpu_add(&p.chunk_flags[j], 1u);
        }
        done_in_chunk = 0;
      }
      if (i + Cfg::COPY_BUFS < total) {
        bulk_wait_read_all();
        ok = issue(i + Cfg::COPY_BUFS);
      }
    }
    if (pieces_per_chunk == 0) {
      for (int s = 0; s < p.n; ++s) {
        if (s == p.rank) {
          const unsigned int prev = atomicAdd(&p.chunk_flags[s], 1u);
          if (prev + 1u == static_cast<unsigned int>(p.epoch) * static_cast<unsigned int>(p.copy_ctas))
            st_release_sys_u64(p.my_ready, p.epoch);
        } else {
          red_release_gpu_add(&p.chunk_flags[s], 1u);
        }
      }
    }
    bulk_wait_all();
    for (int b = 0; b < Cfg::COPY_BUFS; ++b)
      if (pending & (1u << b)) mbar_wait(&bars[b], (pend_parity >> b) & 1u, nullptr, 0);
  }
  __syncthreads();

  // ------------------------------------------------------------ GEMM phase (every CTA)
  const int mt_chunk = p.T_local / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int tpc = mt_chunk * num_n;
  const unsigned int want = static_cast<unsigned int>(p.epoch) * static_cast<unsigned int>(p.copy_ctas);
  int ready_mask = 0;
  auto tile_of = [&](int t, int& mb, int& nb, int& chunk) { rotated_tile(t, tpc, mt_chunk, p.n, p.rank, 0, mb, nb, chunk); };
  auto wait_chunk = [&](int chunk) -> bool {
    if (chunk == p.rank) return true;  // own tiles read x_local directly
    if (ready_mask & (1 << chunk)) return true;
    const unsigned int* f = &p.chunk_flags[chunk];
    if (!spin_until([&] { return static_cast<int>(ld_acquire_gpu_u32(f) - want) >= 0; }, p.status,
                    kStatusTimeoutFlag))
      return false;
    fence_proxy_async_global();
    ready_mask |= 1 << chunk;
    return true;
  };
  auto store = [&](uint32_t t_row, int row, int mb, int nb, int chunk) {
    const long m = static_cast<long>(mb) * BM + row;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(t_row + c, r);
      const int n0 = nb * BN + c;
      if (m >= p.M || n0 >= p.N) continue;
      bf16* crow = p.C + m * p.ldc + n0;
      if (n0 + 32 <= p.N) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          float v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u)
            v[u] = __uint_as_float(r[j + u]) + (p.bias ? __bfloat162float(p.bias[n0 + j + u]) : 0.f);
          uint4 o;
          o.x = pack_bf16x2(v[0], v[1]);
          o.y = pack_bf16x2(v[2], v[3]);
          o.z = pack_bf16x2(v[4], v[5]);
          o.w = pack_bf16x2(v[6], v[7]);
          *reinterpret_cast<uint4*>(crow + j) = o;
        }
      } else {
        for (int j = 0; j < 32 && n0 + j < p.N; ++j)
          crow[j] = __float2bfloat16(__uint_as_float(r[j]) + (p.bias ? __bfloat162float(p.bias[n0 + j]) : 0.f));
      }
    }
  };
  auto published = [&](int) {};
  gemm_phase<BN, B_MN, false>(sm, tmem_base, &tmA, &tmB, p.K, tpc * p.n, p.tile_ctr, p.status, tile_of, wait_chunk, store,
                       published, &tmA_local, p.rank, mt_chunk);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ================================================================== GEMM + RS
template <int BN, bool B_MN>
__global__ void __launch_bounds__(192, 1)
    gemm_rs_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, RsParams p) {
  using Cfg = FusedCfg<BN>;
  constexpr int BM = Cfg::BM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  FusedSmem<BN> sm(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt_chunk = p.T_local / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int tpc = mt_chunk * num_n;

  if (threadIdx.x == 0) sm.init();
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(sm.tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *sm.tmem_slot;

  auto tile_of = [&](int t, int& mb, int& nb, int& chunk) { rotated_tile(t, tpc, mt_chunk, p.n, p.rank, 1, mb, nb, chunk); };
  auto wait_chunk = [&](int) -> bool { return true; };
  auto store = [&](uint32_t t_row, int row, int mb, int nb, int chunk) {
    const long m_loc = static_cast<long>(mb - chunk * mt_chunk) * BM + row;
    bf16* dst_base = p.peer_recv[chunk] + (static_cast<long>(p.rank) * p.T_local + m_loc) * p.N;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(t_row + c, r);
      const int n0 = nb * BN + c;
      if (n0 >= p.N) continue;
      bf16* drow = dst_base + n0;
      if (n0 + 32 <= p.N) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 o;
          o.x = pack_bf16x2(__uint_as_float(r[j + 0]), __uint_as_float(r[j + 1]));
          o.y = pack_bf16x2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          o.z = pack_bf16x2(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5]));
          o.w = pack_bf16x2(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7]));
          *reinterpret_cast<uint4*>(drow + j) = o;
        }
      } else {
        for (int j = 0; j < 32 && n0 + j < p.N; ++j) drow[j] = __float2bfloat16(__uint_as_float(r[j]));
      }
    }
  };
  auto published = [&](int chunk) { red_release_sys_add(p.peer_counter[chunk], 1u); };
  gemm_phase<BN, B_MN, true>(sm, tmem_base, &tmA, &tmB, p.K, tpc * p.n, p.tile_ctr, p.status, tile_of, wait_chunk, store,
                       published);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }

  // ------------------------------------------------------------ reduction of this rank's chunk
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const unsigned int want = static_cast<unsigned int>(tpc * p.n);
    const unsigned int* ctr = p.my_counter;
    s_ok = spin_until([&] { return ld_acquire_sys_u32(ctr) >= want; }, p.status, kStatusTimeoutPeer) ? 1 : 0;
  }
  __syncthreads();
  if (s_ok) {
    const int64_t vec_per_row = p.N / 8;
    const int64_t total = static_cast<int64_t>(p.T_local) * vec_per_row;
    const int64_t slot = static_cast<int64_t>(p.T_local) * p.N;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t r = i / vec_per_row, cv = i % vec_per_row;
      float acc8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int s = 0; s < p.n; ++s) {
        const uint4 u = *reinterpret_cast<const uint4*>(p.my_recv + s * slot + r * p.N + cv * 8);
        acc8[0] += bf16_lo(u.x); acc8[1] += bf16_hi(u.x); acc8[2] += bf16_lo(u.y); acc8[3] += bf16_hi(u.y);
        acc8[4] += bf16_lo(u.z); acc8[5] += bf16_hi(u.z); acc8[6] += bf16_lo(u.w); acc8[7] += bf16_hi(u.w);
      }
      if (p.bias) {
#pragma unroll
        for (int u = 0; u < 8; ++u) acc8[u] += __bfloat162float(p.bias[cv * 8 + u]);
      }
      uint4 o;
      o.x = pack_bf16x2(acc8[0], acc8[1]);
      o.y = pack_bf16x2(acc8[2], acc8[3]);
      o.z = pack_bf16x2(acc8[4], acc8[5]);
      o.w = pack_bf16x2(acc8[6], acc8[7]);
      *reinterpret_cast<uint4*>(p.out + r * p.ldo + cv * 8) = o;
    }
  }
  // The last block out rewinds this parity's counter pair for its next use.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(p.my_counter + 1, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(p.my_counter, 0u);
      atomicExch(p.my_counter + 1, 0u);
      __threadfence_system();
    }
  }
}

// ================================================================== host launchers
// Ordinary launch: no wait in these kernels depends on a CTA that may not be
// resident yet - copy CTAs (lowest indices) never wait on GEMM CTAs, and the
// dynamic tile counter lets whichever CTAs are running drain every tile
// before any CTA enters a phase that waits for all tiles.
template <typename Kern>
static void coop_launch(Kern kern, int grid, int smem, void** args, cudaStream_t stream) {
  static bool attr_done = false;
  if (!attr_done) {
    NTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_done = true;
  }
  NTB_CUDA_CHECK(cudaLaunchKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(192), args,
                                  static_cast<size_t>(smem), stream));
  NTB_LAUNCH_CHECK(1);
}

// x_full_out: [n*T_local, K] local buffer (receives the gathered X; A operand)
// slots: int64 [n] device addresses of every rank's shard slot for this epoch
// ready: int64 [n] device addresses of every rank's ready word; my_ready = ready[rank]
// chunk_flags: int32 [n] local counters
void ag_gemm(const at::Tensor& x_local, at::Tensor& x_full_out, const at::Tensor& w, at::Tensor& y,
             const c10::optional<at::Tensor>& bias, bool b_mn, std::vector<int64_t> slots, std::vector<int64_t> ready,
             at::Tensor& chunk_flags, at::Tensor& tile_ctr, int64_t rank, int64_t epoch, int64_t copy_ctas) {
  const int n = static_cast<int>(slots.size());
  TORCH_CHECK(n >= 1 && n <= kMaxRanks && static_cast<int>(ready.size()) == n, "ag_gemm: 1..8 ranks");
  TORCH_CHECK(x_full_out.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "ag_gemm: bf16");
  TORCH_CHECK(x_full_out.is_contiguous() && w.stride(1) == 1 && y.is_contiguous(), "ag_gemm: layouts");
  const int64_t M = x_full_out.size(0), K = x_full_out.size(1);
  TORCH_CHECK(M % n == 0 && (M / n) % 128 == 0, "ag_gemm: rows per rank must be a multiple of 128");
  const int64_t N = b_mn ? w.size(1) : w.size(0);
  TORCH_CHECK((b_mn ? w.size(0) : w.size(1)) == K, "ag_gemm: K mismatch");
  TORCH_CHECK(y.size(0) == M && y.size(1) == N && y.scalar_type() == at::kBFloat16, "ag_gemm: out");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "ag_gemm: K, N multiples of 8");
  AgParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.T_local = static_cast<int>(M / n);
  p.n = n;
  p.rank = static_cast<int>(rank);
  p.copy_ctas = static_cast<int>(copy_ctas);
  p.epoch = static_cast<unsigned long long>(epoch);
  p.full = reinterpret_cast<bf16*>(x_full_out.data_ptr());
  TORCH_CHECK(x_local.is_contiguous() && x_local.scalar_type() == at::kBFloat16 && x_local.size(0) == M / n &&
                  x_local.size(1) == K,
              "ag_gemm: local shard shape");
  p.x_local = reinterpret_cast<const bf16*>(x_local.data_ptr());
  p.my_slot = reinterpret_cast<bf16*>(slots[rank]);
  for (int i = 0; i < n; ++i) {
    p.peer_slot[i] = reinterpret_cast<const bf16*>(slots[i]);
    p.peer_ready[i] = reinterpret_cast<const unsigned long long*>(ready[i]);
  }
  p.my_ready = reinterpret_cast<unsigned long long*>(ready[rank]);
  p.chunk_flags = reinterpret_cast<unsigned int*>(chunk_flags.data_ptr());
  p.tile_ctr = reinterpret_cast<unsigned int*>(tile_ctr.data_ptr());
  p.C = reinterpret_cast<bf16*>(y.data_ptr());
  p.ldc = y.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const bf16*>(bias->data_ptr()) : nullptr;
  p.status = device_status(x_full_out.get_device());
  const int dev = x_full_out.get_device();
  const int grid = num_sms(dev);
  TORCH_CHECK(p.copy_ctas >= 1 && p.copy_ctas < grid, "ag_gemm: copy CTA count");
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  TmaSlots& ts = tls_tma_slots();
  const bool wide = N > 128;
  make_tma_2d_bf16(&ts.m[0], x_full_out.data_ptr(), K, M, K, 64, 128);
  make_tma_2d_bf16(&ts.m[1], w.data_ptr(), w.size(1), w.size(0), w.stride(0), 64, b_mn ? 64 : (wide ? 256 : 128));
  make_tma_2d_bf16(&ts.m[2], x_local.data_ptr(), K, M / n, K, 64, 128);
  NTB_CUDA_CHECK(cudaMemsetAsync(tile_ctr.data_ptr(), 0, sizeof(unsigned int), stream));
  void* args[4] = {&ts.m[0], &ts.m[1], &ts.m[2], &p};
  if (wide) {
    if (b_mn) coop_launch(ag_gemm_kernel<256, true>, grid, FusedCfg<256>::SMEM_BYTES, args, stream);
    else coop_launch(ag_gemm_kernel<256, false>, grid, FusedCfg<256>::SMEM_BYTES, args, stream);
  } else {
    if (b_mn) coop_launch(ag_gemm_kernel<128, true>, grid, FusedCfg<128>::SMEM_BYTES, args, stream);
    else coop_launch(ag_gemm_kernel<128, false>, grid, FusedCfg<128>::SMEM_BYTES, args, stream);
  }
}

// x: [n*T_local, K] local operand; out: [T_local, N]
// recv: int64 [n] device addresses of every rank's receive slot base for this epoch ([n][T_local][N] bf16)
// counters: int64 [n] device addresses of every rank's counter pair for this epoch parity
void gemm_rs(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, const c10::optional<at::Tensor>& bias,
             bool b_mn, std::vector<int64_t> recv, std::vector<int64_t> counters, at::Tensor& tile_ctr, int64_t rank,
             int64_t epoch) {
  const int n = static_cast<int>(recv.size());
  TORCH_CHECK(n >= 1 && n <= kMaxRanks && static_cast<int>(counters.size()) == n, "gemm_rs: 1..8 ranks");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm_rs: bf16");
  TORCH_CHECK(x.is_contiguous() && w.stride(1) == 1 && out.is_contiguous(), "gemm_rs: layouts");
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(M % n == 0 && (M / n) % 128 == 0, "gemm_rs: rows per rank must be a multiple of 128");
  const int64_t N = b_mn ? w.size(1) : w.size(0);
  TORCH_CHECK((b_mn ? w.size(0) : w.size(1)) == K, "gemm_rs: K mismatch");
  TORCH_CHECK(out.size(0) == M / n && out.size(1) == N, "gemm_rs: out");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "gemm_rs: K, N multiples of 8");
  RsParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.T_local = static_cast<int>(M / n);
  p.n = n;
  p.rank = static_cast<int>(rank);
  p.epoch = static_cast<unsigned long long>(epoch);
  for (int i = 0; i < n; ++i) {
    p.peer_recv[i] = reinterpret_cast<bf16*>(recv[i]);
    p.peer_counter[i] = reinterpret_cast<unsigned int*>(counters[i]);
  }
  p.my_counter = reinterpret_cast<unsigned int*>(counters[rank]);
  p.my_recv = reinterpret_cast<const bf16*>(recv[rank]);
  p.tile_ctr = reinterpret_cast<unsigned int*>(tile_ctr.data_ptr());
  p.out = reinterpret_cast<bf16*>(out.data_ptr());
  p.ldo = out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const bf16*>(bias->data_ptr()) : nullptr;
  p.status = device_status(x.get_device());
  const int dev = x.get_device();
  const int grid = num_sms(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  TmaSlots& ts = tls_tma_slots();
  const bool wide = N > 128;
  make_tma_2d_bf16(&ts.m[2], x.data_ptr(), K, M, x.stride(0), 64, 128);
  make_tma_2d_bf16(&ts.m[3], w.data_ptr(), w.size(1), w.size(0), w.stride(0), 64, b_mn ? 64 : (wide ? 256 : 128));
  NTB_CUDA_CHECK(cudaMemsetAsync(tile_ctr.data_ptr(), 0, sizeof(unsigned int), stream));
  void* args[3] = {&ts.m[2], &ts.m[3], &p};
  if (wide) {
    if (b_mn) coop_launch(gemm_rs_kernel<256, true>, grid, FusedCfg<256>::SMEM_BYTES, args, stream);
    else coop_launch(gemm_rs_kernel<256, false>, grid, FusedCfg<256>::SMEM_BYTES, args, stream);
  } else {
    if (b_mn) coop_launch(gemm_rs_kernel<128, true>, grid, FusedCfg<128>::SMEM_BYTES, args, stream);
    else coop_launch(gemm_rs_kernel<128, false>, grid, FusedCfg<128>::SMEM_BYTES, args, stream);
  }
}

}  // namespace ntb
