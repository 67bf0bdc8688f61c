// Fused tensor-parallel compute + collective kernels over NVLink peer memory.
//
// ag_gemm:  Y[T, N] = AllGather_T(X_shard)[T, K] . op(W)^T        (ColumnParallel fwd,
//           also returns the gathered X for the weight gradient)   RowParallel bwd dgrad)
// gemm_rs:  Y_shard[T/n, N] = ReduceScatter_T(X[T, K] . op(W)^T)  (RowParallel fwd,
//                                                                   ColumnParallel bwd dgrad)
//
// Both are ONE launch of persistent CTAs (one per SM) on every rank of the
// tensor-parallel group; the GEMM core is the same tcgen05/TMA/TMEM pipeline
// as gemm.cu (128 x BN x 64 tiles, 2 TMEM accumulators, warp roles
// TMA / MMA / 4 epilogue warps). Tiles are handed out by a global atomic
// counter, so whichever CTAs are resident drain all the work and no wait
// depends on a CTA that has not started.
//
// ag_gemm: tiles run chunk by chunk in rank-rotated order, own chunk first
// (its A operand is read straight from the local shard). Two copy warps per
// CTA, next to the GEMM's six, gather X while the GEMM runs (the epilogue
// warps stay free to drain accumulators): they claim 16 KB pieces from a
// second atomic counter - the
// own shard first (local -> gathered buffer + this rank's symmetric slot),
// then every peer's shard from its symmetric slot (peer loads over NVLink ->
// gathered buffer). The warp that completes the own shard publishes the epoch
// in this rank's ready word (system-scope release); a peer piece is read only
// after the owner's ready word shows the epoch. Each finished piece bumps a
// local per-chunk counter, and the TMA producer waits on it before the first A
// load of a peer chunk, so tiles of chunk j overlap the copy of chunk j+1.
//
// gemm_rs: tiles run by destination chunk, peers first, own chunk last. A
// peer-chunk tile is converted to bf16 and written as whole 128-byte row
// segments into the destination's receive slot for this source rank, then
// (system-scope fence) one thread adds 1 to the destination's arrival counter
// of that tile. An own-chunk tile waits (bounded) until its n-1 peer partials
// have arrived and writes sum(peer partials) + own accumulator (+ bias) as the
// final output: the reduction is fused into the epilogue, no separate pass.
//
// Buffers alternate between two slots by epoch parity; a rank reuses a slot
// only two calls later, by which time every peer has finished the call that
// read it (each call waits on every peer's data of the previous epoch).
// Every wait is bounded and reports through the status word.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"
#include "peer.cuh"

#include <mutex>
#include <set>
#include <utility>

namespace ntb {

using bf16 = __nv_bfloat16;
constexpr int kMaxRanks = 8;

// ------------------------------------------------------------------ shared GEMM core
template <int BN>
struct FusedCfg {
  static constexpr int BM = 128, BK = 64, STAGES = (BN == 256) ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int STAGE_BYTES = 4 * 4096;  // epilogue staging: 4 KB per epilogue warp
  static constexpr int SMEM_BYTES = 1024 + STAGES * (A_BYTES + B_BYTES) + STAGE_BYTES + 512;
};

constexpr int kAgPiece = 16384;  // bytes of X claimed per copy step by one epilogue warp

struct AgParams {
  int M, N, K;          // M = n * T_local
  int T_local, n, rank;
  unsigned long long epoch;
  bf16* full;                                  // local gathered X [M, K]
  const bf16* x_local;                         // this rank's shard [T_local, K]
  bf16* my_slot;                               // this rank's symmetric slot for this epoch
  const bf16* peer_slot[kMaxRanks];            // each rank's shard slot [T_local, K] (this epoch)
  const unsigned long long* peer_ready[kMaxRanks];
  unsigned long long* my_ready;
  unsigned int* ctr;                           // local: [0] tile counter, [1] piece counter (zeroed per call)
  unsigned long long* chunk_done;              // local [n]: pieces copied per chunk (zeroed per call)
  bf16* C;
  long ldc;
  const bf16* bias;
  int* status;
  unsigned long long* trace;                   // optional [grid][8] globaltimer stamps (nullptr: off)
};

struct RsParams {
  int M, N, K;          // M = n * T_local (full rows of the partial product)
  int T_local, n, rank;
  unsigned long long epoch;
  bf16* peer_recv[kMaxRanks];                  // each rank's receive slot base [n][T_local][N] (this epoch)
  unsigned int* peer_tctr[kMaxRanks];          // each rank's per-tile arrival counters (this epoch parity)
  unsigned int* my_tctr;
  const bf16* my_recv;
  unsigned int* ctr;                           // local: [0] tile counter (zeroed per call)
  bf16* out;                                   // [T_local, N]
  long ldo;
  const bf16* bias;
  int* status;
  unsigned long long* trace;                   // optional [grid][8] globaltimer stamps (nullptr: off)
};

// Timeline stamps (ns, %globaltimer) per CTA when tracing is on:
//   0 start   1 AG gather done (warp 2)   2 first tile handed out   3 first remote-chunk wait done
//   4 producer out of tiles   5 last epilogue tile stored   6 AG own shard published   7 end
__device__ __forceinline__ void stamp(unsigned long long* trace, int ev) {
  if (trace != nullptr) trace[blockIdx.x * 8 + ev] = globaltimer_ns();
}

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
//   epilogue staging (4 x 4 KB)
//   barriers: full[S] empty[S] tfull[2] tempty[2] tdone[4] drain tring_full[4] tring_empty[4]
//   tile ring int[4], TMEM base slot
template <int BN>
struct FusedSmem {
  using Cfg = FusedCfg<BN>;
  uint8_t* sA;
  uint8_t* sB;
  uint8_t* stage;
  uint64_t *full, *empty, *tfull, *tempty, *tdone, *drain, *tring_full, *tring_empty;
  int* tring;
  uint32_t* tmem_slot;
  __device__ __forceinline__ explicit FusedSmem(uint8_t* smem) {
    sA = smem;
    sB = smem + Cfg::STAGES * Cfg::A_BYTES;
    stage = sB + Cfg::STAGES * Cfg::B_BYTES;
    full = reinterpret_cast<uint64_t*>(stage + Cfg::STAGE_BYTES);
    empty = full + Cfg::STAGES;
    tfull = empty + Cfg::STAGES;
    tempty = tfull + 2;
    tdone = tempty + 2;
    drain = tdone + 4;
    tring_full = drain + 1;
    tring_empty = tring_full + 4;
    tring = reinterpret_cast<int*>(tring_empty + 4);
    tmem_slot = reinterpret_cast<uint32_t*>(tring + 4);
  }
  // publisher: a seventh warp releases every finished tile to its destination (reduce-scatter);
  // ring slots then also wait for it.
  __device__ __forceinline__ void init(bool publisher) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&tdone[b], 128);
      mbar_init(&tring_full[b], 1);
      mbar_init(&tring_empty[b], publisher ? 129 : 128);
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
};

// Warp-cooperative epilogue store. The calling warp owns TMEM lanes [32q, 32q+32)
// (tile rows) and BN fp32 accumulator columns at `t_row`. Each 64-column group is
// converted to bf16, staged through the warp's 4 KB of shared memory (16-byte
// chunks XOR-swizzled by row to avoid bank conflicts) and written out as whole
// 128-byte row segments: one warp instruction covers 4 rows x 128 B, so stores to
// peer memory cross NVLink as full lines instead of 16-byte pieces.
//   dst0   destination of the warp's first row at the tile's first column; ld its row stride
//   ncols  valid columns from the tile start (a multiple of 8)
//   bias   optional, indexed from the tile's first column
//   part0  optional: partial products to add, source s at part0 + s * part_stride
//          (row stride part_ld), for s in [0, nparts) except `skip` (reduce-scatter epilogue)
//   facc0  optional: an fp32 sum of partials to add (row stride facc_ld); each value read is
//          set back to zero, so the buffer is zero at rest again after the tile
template <int BN>
__device__ __forceinline__ void warp_store_tile(uint32_t t_row, uint8_t* stage, bf16* dst0, long ld, int ncols,
                                                const bf16* bias, const bf16* part0 = nullptr, long part_ld = 0,
                                                long part_stride = 0, int nparts = 0, int skip = -1,
                                                float* facc0 = nullptr, long facc_ld = 0) {
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int g = 0; g < BN; g += 64) {
    if (g >= ncols) break;  // warp-uniform
    uint32_t r0[32], r1[32];
    tmem_ld32(t_row + g, r0);
    tmem_ld32(t_row + g + 32, r1);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 o;
      uint32_t* w = &o.x;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t a = j < 4 ? r0[j * 8 + 2 * u] : r1[(j - 4) * 8 + 2 * u];
        const uint32_t b = j < 4 ? r0[j * 8 + 2 * u + 1] : r1[(j - 4) * 8 + 2 * u + 1];
        w[u] = pack_bf16x2(__uint_as_float(a), __uint_as_float(b));
      }
      *reinterpret_cast<uint4*>(stage + lane * 128 + ((j ^ (lane & 7)) * 16)) = o;
    }
    __syncwarp();
    const int chunk = lane & 7;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int row = it * 4 + (lane >> 3);
      const int c = g + chunk * 8;
      if (c >= ncols) continue;
      uint4 v = *reinterpret_cast<const uint4*>(stage + row * 128 + ((chunk ^ (row & 7)) * 16));
      if (bias != nullptr || part0 != nullptr || facc0 != nullptr) {
        float acc[8] = {bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y),
                        bf16_lo(v.z), bf16_hi(v.z), bf16_lo(v.w), bf16_hi(v.w)};
        if (facc0 != nullptr) {
          float4* f = reinterpret_cast<float4*>(facc0 + row * facc_ld + c);
          const float4 f0 = f[0], f1 = f[1];
          acc[0] += f0.x; acc[1] += f0.y; acc[2] += f0.z; acc[3] += f0.w;
          acc[4] += f1.x; acc[5] += f1.y; acc[6] += f1.z; acc[7] += f1.w;
          f[0] = make_float4(0.f, 0.f, 0.f, 0.f);
          f[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (part0 != nullptr) {
          for (int s = 0; s < nparts; ++s) {
            if (s == skip) continue;
            const uint4 u = *reinterpret_cast<const uint4*>(part0 + s * part_stride + row * part_ld + c);
            acc[0] += bf16_lo(u.x); acc[1] += bf16_hi(u.x); acc[2] += bf16_lo(u.y); acc[3] += bf16_hi(u.y);
            acc[4] += bf16_lo(u.z); acc[5] += bf16_hi(u.z); acc[6] += bf16_lo(u.w); acc[7] += bf16_hi(u.w);
          }
        }
        if (bias != nullptr) {
#pragma unroll
          for (int u = 0; u < 8; ++u) acc[u] += __bfloat162float(bias[c + u]);
        }
        v.x = pack_bf16x2(acc[0], acc[1]);
        v.y = pack_bf16x2(acc[2], acc[3]);
        v.z = pack_bf16x2(acc[4], acc[5]);
        v.w = pack_bf16x2(acc[6], acc[7]);
      }
      *reinterpret_cast<uint4*>(dst0 + row * ld + c) = v;
    }
    __syncwarp();
  }
}

// Runs GEMM tiles handed out by a global atomic counter. `tile_of(t, mb, nb, chunk)` maps
// a tile index; `wait_chunk(chunk)` (producer) gates A loads; `pre_epilogue()` runs once in
// every epilogue warp before its first tile; `store(t_row, mb, nb, chunk)` is the per-tile
// epilogue of one warp (its 32 TMEM lanes); `published(mb, nb, chunk)` runs once per tile in
// one thread after all epilogue threads stored (and, for chunks other than `own_chunk`,
// fenced at system scope). Own-chunk tiles read A through `tmA_own` when it is given.
template <int BN, bool B_MN, bool PUBLISH, typename TileOf, typename WaitChunk, typename PreEpi, typename Store,
          typename Published>
__device__ __forceinline__ void gemm_phase(FusedSmem<BN>& sm, uint32_t tmem_base, const CUtensorMap* tmA,
                                           const CUtensorMap* tmB, int K, int num_tiles, unsigned int* tile_ctr,
                                           int* status, TileOf tile_of, WaitChunk wait_chunk, PreEpi pre_epilogue,
                                           Store store, Published published, unsigned long long* trace,
                                           const CUtensorMap* tmA_own, int own_chunk, int mtiles_per_chunk) {
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
      bool first_remote_stamped = false;
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
        if (tt < 0) {
          stamp(trace, 4);
          break;
        }
        if (i == 0) stamp(trace, 2);
        int mb, nb, chunk;
        tile_of(tt, mb, nb, chunk);
        if (!wait_chunk(chunk)) break;
        if (chunk != own_chunk && !first_remote_stamped) {
          stamp(trace, 3);
          first_remote_stamped = true;
        }
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
  } else if (warp == 6) {
    // Publisher (reduce-scatter only): per tile, in ring order, wait until the epilogue stored it,
    // then one system-scope fence + the arrival increment at the destination.
    if constexpr (PUBLISH) {
      if (lane == 0) {
        for (int i = 0;; ++i) {
          const int slot = i & 3;
          const uint32_t par = static_cast<uint32_t>((i >> 2) & 1);
          if (!mbar_wait(&sm.tring_full[slot], par, status, kStatusTimeoutEpilogue)) break;
          const int t = sm.tring[slot];
          if (t < 0) break;
          int mb, nb, chunk;
          tile_of(t, mb, nb, chunk);
          if (!mbar_wait(&sm.tdone[slot], par, status, kStatusTimeoutEpilogue)) break;
          published(mb, nb, chunk);
          mbar_arrive(&sm.tring_empty[slot]);
        }
      }
    }
  } else {
    const int q = warp & 3;
    pre_epilogue();
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int i = 0;; ++i) {
      const int slot = i & 3;
      const uint32_t par = static_cast<uint32_t>((i >> 2) & 1);
      if (!mbar_wait(&sm.tring_full[slot], par, status, kStatusTimeoutEpilogue)) break;
      const int t = sm.tring[slot];
      if (t < 0) {
        if (warp == 2 && lane == 0) stamp(trace, 5);
        break;
      }
      int mb, nb, chunk;
      tile_of(t, mb, nb, chunk);
      if (!mbar_wait(&sm.tfull[acc], acc_phase, status, kStatusTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      store(t_row, mb, nb, chunk);
      tc_fence_before();
      mbar_arrive(&sm.tempty[acc]);
      // Stores of this tile are done (mbarrier arrive = CTA-scope release); the publisher
      // warp makes them visible system-wide and signals the destination.
      if constexpr (PUBLISH) mbar_arrive(&sm.tdone[slot]);
      mbar_arrive(&sm.tring_empty[slot]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
}

// ================================================================== AG + GEMM
constexpr int kAgCopyWarps = 2;

template <int BN, bool B_MN>
__global__ void __launch_bounds__(192 + 32 * kAgCopyWarps, 1)
    ag_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA_local, AgParams p) {
  using Cfg = FusedCfg<BN>;
  constexpr int BM = Cfg::BM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  FusedSmem<BN> sm(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) sm.init(false);
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
  if (threadIdx.x == 0) stamp(p.trace, 0);

  const int mt_chunk = p.T_local / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int tpc = mt_chunk * num_n;
  const long chunk_bytes = static_cast<long>(p.T_local) * p.K * 2;
  const int ppc = static_cast<int>((chunk_bytes + kAgPiece - 1) / kAgPiece);  // pieces per chunk
  int ready_mask = 0;
  auto tile_of = [&](int t, int& mb, int& nb, int& chunk) { rotated_tile(t, tpc, mt_chunk, p.n, p.rank, 0, mb, nb, chunk); };
  auto wait_chunk = [&](int chunk) -> bool {
    if (chunk == p.rank) return true;  // own tiles read x_local directly
    if (ready_mask & (1 << chunk)) return true;
    const unsigned long long* f = &p.chunk_done[chunk];
    const unsigned long long want = static_cast<unsigned long long>(ppc);
    if (!spin_until([&] { return ld_acquire_gpu_u64(f) >= want; }, p.status, kStatusTimeoutFlag)) return false;
    fence_proxy_async_global();  // generic-proxy writes of the gather -> TMA (async proxy) reads
    ready_mask |= 1 << chunk;
    return true;
  };
  // Gather of X by the epilogue warps (see the file comment).
  auto pre_epilogue = [&]() {
    int waited = 0;
    while (true) {
      int idx = 0;
      if (lane == 0) idx = static_cast<int>(atomicAdd(p.ctr + 1, 1u));
      idx = __shfl_sync(0xffffffffu, idx, 0);
      if (idx >= ppc * p.n) break;
      const int s = idx / ppc, j = (p.rank + s) % p.n;
      const long off = static_cast<long>(idx % ppc) * kAgPiece;
      const int nvec = static_cast<int>(min(static_cast<long>(kAgPiece), chunk_bytes - off) / 16);
      if (j != p.rank && !(waited & (1 << j))) {
        int ok = 1;
        if (lane == 0) {
          const unsigned long long* rw = p.peer_ready[j];
          const unsigned long long want = p.epoch;
          ok = spin_until([&] { return ld_acquire_sys_u64(rw) >= want; }, p.status, kStatusTimeoutPeer) ? 1 : 0;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        (void)ld_acquire_sys_u64(p.peer_ready[j]);  // every lane acquires before reading the peer's slot
        waited |= 1 << j;
      }
      const uint4* src = reinterpret_cast<const uint4*>(
          reinterpret_cast<const uint8_t*>(j == p.rank ? p.x_local : p.peer_slot[j]) + off);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.full + static_cast<long>(j) * p.T_local * p.K) + off);
      uint4* dst2 = j == p.rank ? reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.my_slot) + off) : nullptr;
#pragma unroll 1
      for (int base = 0; base < nvec; base += 32 * 16) {
        uint4 v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int i = base + u * 32 + lane;
          if (i < nvec) v[u] = src[i];
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int i = base + u * 32 + lane;
          if (i < nvec) {
            dst[i] = v[u];
            if (dst2 != nullptr) dst2[i] = v[u];
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        if (j == p.rank) {
          __threadfence_system();
          const unsigned long long prev = atomicAdd(&p.chunk_done[j], 1ull);
          if (prev + 1 == static_cast<unsigned long long>(ppc)) {
            // This warp completed the own shard: publish the epoch to the peers.
            __threadfence_system();
            st_release_sys_u64(p.my_ready, p.epoch);
            stamp(p.trace, 6);
          }
        } else {
          __threadfence();
          atomicAdd(&p.chunk_done[j], 1ull);
        }
      }
    }
    if (warp == 6 && lane == 0) stamp(p.trace, 1);
  };
  auto store = [&](uint32_t t_row, int mb, int nb, int) {
    const int q = warp & 3;
    const long m0 = static_cast<long>(mb) * BM + q * 32;  // rows always in range: M = n * T_local, T_local % 128 == 0
    const int n0 = nb * BN;
    warp_store_tile<BN>(t_row, sm.stage + q * 4096, p.C + m0 * p.ldc + n0, p.ldc, p.N - n0,
                        p.bias != nullptr ? p.bias + n0 : nullptr);
  };
  auto published = [&](int, int, int) {};
  auto nothing = [&]() {};
  if (warp >= 6) {
    pre_epilogue();  // the copy warps: the gather of X
  } else {
    gemm_phase<BN, B_MN, false>(sm, tmem_base, &tmA, &tmB, p.K, tpc * p.n, p.ctr, p.status, tile_of, wait_chunk,
                                nothing, store, published, p.trace, &tmA_local, p.rank, mt_chunk);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  if (threadIdx.x == 0) stamp(p.trace, 7);
}

// ================================================================== GEMM + RS
template <int BN, bool B_MN>
__global__ void __launch_bounds__(224, 1)
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

  if (threadIdx.x == 0) sm.init(true);
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
  if (threadIdx.x == 0) stamp(p.trace, 0);

  const long slot_elems = static_cast<long>(p.T_local) * p.N;
  auto tile_of = [&](int t, int& mb, int& nb, int& chunk) { rotated_tile(t, tpc, mt_chunk, p.n, p.rank, 1, mb, nb, chunk); };
  auto wait_chunk = [&](int) -> bool { return true; };
  auto pre_epilogue = [&]() {};
  auto store = [&](uint32_t t_row, int mb, int nb, int chunk) {
    const int q = warp & 3;
    const int lm = mb - chunk * mt_chunk;
    const long m_loc = static_cast<long>(lm) * BM + q * 32;
    const int n0 = nb * BN;
    if (chunk != p.rank) {
      bf16* dst0 = p.peer_recv[chunk] + (static_cast<long>(p.rank) * p.T_local + m_loc) * p.N + n0;
      warp_store_tile<BN>(t_row, sm.stage + q * 4096, dst0, p.N, p.N - n0, nullptr);
    } else {
      const unsigned int* tc = p.my_tctr + nb * mt_chunk + lm;
      const unsigned int want = static_cast<unsigned int>(p.n - 1);
      int ok = 1;
      if (lane == 0) ok = spin_until([&] { return ld_acquire_sys_u32(tc) >= want; }, p.status, kStatusTimeoutPeer) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) return;
      (void)ld_acquire_sys_u32(tc);  // every lane acquires before reading the peers' partials
      warp_store_tile<BN>(t_row, sm.stage + q * 4096, p.out + m_loc * p.ldo + n0, p.ldo, p.N - n0,
                          p.bias != nullptr ? p.bias + n0 : nullptr, p.my_recv + m_loc * p.N + n0, p.N, slot_elems,
                          p.n, p.rank);
    }
  };
  auto published = [&](int mb, int nb, int chunk) {
    const int idx = nb * mt_chunk + (mb - chunk * mt_chunk);
    if (chunk != p.rank) {
      __threadfence_system();  // the tile's remote stores (ordered before via the tdone barrier)
      red_release_sys_add(p.peer_tctr[chunk] + idx, 1u);
    } else {
      p.my_tctr[idx] = 0u;  // consumed: rewind for this parity's next use (two calls later)
    }
  };
  gemm_phase<BN, B_MN, true>(sm, tmem_base, &tmA, &tmB, p.K, tpc * p.n, p.ctr, p.status, tile_of, wait_chunk,
                             pre_epilogue, store, published, p.trace, nullptr, p.rank, mt_chunk);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  if (threadIdx.x == 0) stamp(p.trace, 7);
}

// ================================================================== GEMM + RS, progressive pull
// Same GEMM and tile order as gemm_rs (destination chunks rank-rotated, this rank's own chunk
// last), but no remote stores: a tile for destination chunk c is stored as bf16 into THIS rank's
// partial slot (local), and the publisher warp releases it with one 8-byte epoch store into the
// destination's ready word for (source, tile). Two more warps per CTA pull: they claim
// (source, tile) items of this rank's own chunk in the order the sources finish them (source
// rank - s computes this rank's chunk at its step s), wait for the ready word, read the tile over
// NVLink and add it into a local fp32 accumulator with red.global.add.v4.f32, then count the
// tile. The own-chunk epilogue (the GEMM's last tiles) waits until every source was added, adds
// the accumulator to its own bf16-rounded tile (+ bias), writes the output and zeroes the
// accumulator tile for the next call. The pulls of early sources overlap the rest of the GEMM.
// Numerics equal the pull reduce-scatter's: each rank's partial is rounded to bf16 once and the
// partials are summed in fp32 (here in arrival order).
constexpr int kRspPullWarps = 2;

struct RspParams {
  int M, N, K;  // M = n * T_local
  int T_local, n, rank, tpc_stride;
  unsigned long long epoch;
  bf16* my_part;                                // this rank's partial slot [n][T_local][N] (local)
  const bf16* peer_part[kMaxRanks];             // every rank's partial slot (peer mappings)
  unsigned long long* peer_rdy[kMaxRanks];      // rank r's ready words for source = this rank [tpc]
  const unsigned long long* my_rdy;             // this rank's ready words [n sources][tpc_stride]
  float* acc;                                   // local fp32 [T_local, N], zero at rest
  unsigned int* acc_cnt;                        // local [tpc]: sources added per tile, zero at rest
  unsigned int* ctr;                            // local: [0] tile counter, [1] pull item counter (zeroed per call)
  bf16* out;                                    // [T_local, N]
  long ldo;
  const bf16* bias;
  int* status;
  unsigned long long* trace;
};

template <int BN>
__device__ __forceinline__ void rsp_pull_loop(const RspParams& p, int mt_chunk, int tpc) {
  const int lane = threadIdx.x & 31;
  const int items = (p.n - 1) * tpc;
  constexpr int CPR = BN / 8;  // 16-byte chunks per tile row
  while (true) {
    int it = 0;
    if (lane == 0) it = static_cast<int>(atomicAdd(p.ctr + 1, 1u));
    it = __shfl_sync(0xffffffffu, it, 0);
    if (it >= items) break;
    const int s = 1 + it / tpc, idx = it - (it / tpc) * tpc;
    const int src = (p.rank - s + p.n) % p.n;
    const unsigned long long* rdy = p.my_rdy + static_cast<long>(src) * p.tpc_stride + idx;
    int ok = 1;
    if (lane == 0) ok = spin_until([&] { return ld_acquire_sys_u64(rdy) >= p.epoch; }, p.status, kStatusTimeoutPeer) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) break;
    (void)ld_acquire_sys_u64(rdy);  // every lane acquires before reading the source's tile
    const int lm = idx % mt_chunk, nb = idx / mt_chunk;
    const bf16* sp = p.peer_part[src] + (static_cast<long>(p.rank) * p.T_local + lm * 128) * p.N + nb * BN;
    float* dp = p.acc + static_cast<long>(lm * 128) * p.N + nb * BN;
#pragma unroll 1
    for (int base = 0; base < 128 * CPR; base += 32 * 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * 32 + lane;
        const int r = i / CPR, c = (i - r * CPR) * 8;
        v[u] = *reinterpret_cast<const uint4*>(sp + static_cast<long>(r) * p.N + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * 32 + lane;
        const int r = i / CPR, c = (i - r * CPR) * 8;
        float* d = dp + static_cast<long>(r) * p.N + c;
        red_add_v4(d, bf16_lo(v[u].x), bf16_hi(v[u].x), bf16_lo(v[u].y), bf16_hi(v[u].y));
        red_add_v4(d + 4, bf16_lo(v[u].z), bf16_hi(v[u].z), bf16_lo(v[u].w), bf16_hi(v[u].w));
      }
    }
    __threadfence();  // this lane's reductions, before the tile's count
    __syncwarp();
    if (lane == 0) atomicAdd(p.acc_cnt + idx, 1u);
  }
}

template <int BN, bool B_MN>
__global__ void __launch_bounds__(224 + 32 * kRspPullWarps, 1)
    gemm_rsp_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ RspParams p) {
  using Cfg = FusedCfg<BN>;
  constexpr int BM = Cfg::BM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  FusedSmem<BN> sm(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt_chunk = p.T_local / BM;
  const int num_n = p.N / BN;
  const int tpc = mt_chunk * num_n;

  if (threadIdx.x == 0) sm.init(true);
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
  if (threadIdx.x == 0) stamp(p.trace, 0);

  if (warp >= 7) {
    rsp_pull_loop<BN>(p, mt_chunk, tpc);
  } else {
    auto tile_of = [&](int t, int& mb, int& nb, int& chunk) {
      rotated_tile(t, tpc, mt_chunk, p.n, p.rank, 1, mb, nb, chunk);
    };
    auto wait_chunk = [&](int) -> bool { return true; };
    auto pre_epilogue = [&]() {};
    auto store = [&](uint32_t t_row, int mb, int nb, int chunk) {
      const int q = warp & 3;
      const int lm = mb - chunk * mt_chunk;
      const long m_loc = static_cast<long>(lm) * BM + q * 32;
      const int n0 = nb * BN;
      if (chunk != p.rank) {
        bf16* dst0 = p.my_part + (static_cast<long>(chunk) * p.T_local + m_loc) * p.N + n0;
        warp_store_tile<BN>(t_row, sm.stage + q * 4096, dst0, p.N, p.N - n0, nullptr);
      } else {
        const unsigned int* cnt = p.acc_cnt + nb * mt_chunk + lm;
        const unsigned int want = static_cast<unsigned int>(p.n - 1);
        int ok = 1;
        if (lane == 0) ok = spin_until([&] { return ld_acquire_gpu_u32(cnt) >= want; }, p.status, kStatusTimeoutPeer) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) return;
        (void)ld_acquire_gpu_u32(cnt);
        warp_store_tile<BN>(t_row, sm.stage + q * 4096, p.out + m_loc * p.ldo + n0, p.ldo, p.N - n0,
                            p.bias != nullptr ? p.bias + n0 : nullptr, nullptr, 0, 0, 0, -1,
                            p.acc + m_loc * p.N + n0, p.N);
      }
    };
    auto published = [&](int mb, int nb, int chunk) {
      const int idx = nb * mt_chunk + (mb - chunk * mt_chunk);
      if (chunk != p.rank) {
        __threadfence_system();  // the tile's local stores, visible to the destination's loads
        st_relaxed_sys_u64(p.peer_rdy[chunk] + idx, p.epoch);
      } else {
        p.acc_cnt[idx] = 0u;  // consumed: zero at rest for the next call
      }
    };
    gemm_phase<BN, B_MN, true>(sm, tmem_base, &tmA, &tmB, p.K, tpc * p.n, p.ctr, p.status, tile_of, wait_chunk,
                               pre_epilogue, store, published, p.trace, nullptr, p.rank, mt_chunk);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  if (threadIdx.x == 0) stamp(p.trace, 7);
}

// ================================================================== host launchers
// Ordinary launch: no wait in these kernels depends on a CTA that may not be
// resident yet - copy pieces and GEMM tiles are claimed dynamically by the CTAs
// that are running, and a tile only waits on pieces or peer tiles claimed earlier.
template <typename Kern>
static void fused_launch(Kern kern, int grid, int smem, void** args, cudaStream_t stream, int threads = 192) {
  // The dynamic shared-memory opt-in is set once per (device, kernel).
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  NTB_CUDA_CHECK(cudaGetDevice(&dev));
  const void* key = reinterpret_cast<const void*>(kern);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (done.insert({dev, key}).second)
      NTB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  }
  NTB_CUDA_CHECK(cudaLaunchKernel(key, dim3(grid), dim3(threads), args, static_cast<size_t>(smem), stream));
  NTB_LAUNCH_CHECK(1);
}

// x_local: [T_local, K] this rank's shard; x_full_out: [n*T_local, K] local buffer (receives the gathered X)
// slots: int64 [n] device addresses of every rank's shard slot for this epoch
// ready: int64 [n] device addresses of every rank's ready word; my_ready = ready[rank]
// ctrs: int64 [1 + n] local scratch (tile/piece counters, per-chunk piece counts), zeroed here per call
void ag_gemm(const at::Tensor& x_local, at::Tensor& x_full_out, const at::Tensor& w, at::Tensor& y,
             const c10::optional<at::Tensor>& bias, bool b_mn, std::vector<int64_t> slots, std::vector<int64_t> ready,
             at::Tensor& ctrs, int64_t rank, int64_t epoch, const c10::optional<at::Tensor>& trace) {
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
  TORCH_CHECK(x_local.is_contiguous() && x_local.scalar_type() == at::kBFloat16 && x_local.size(0) == M / n &&
                  x_local.size(1) == K,
              "ag_gemm: local shard shape");
  TORCH_CHECK(ctrs.scalar_type() == at::kLong && ctrs.numel() >= 1 + n && ctrs.is_contiguous(), "ag_gemm: ctrs");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x_local.data_ptr()) % 16 == 0 && slots[rank] % 16 == 0,
              "ag_gemm: 16-byte aligned shard and slot");
  AgParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.T_local = static_cast<int>(M / n);
  p.n = n;
  p.rank = static_cast<int>(rank);
  p.epoch = static_cast<unsigned long long>(epoch);
  p.full = reinterpret_cast<bf16*>(x_full_out.data_ptr());
  p.x_local = reinterpret_cast<const bf16*>(x_local.data_ptr());
  p.my_slot = reinterpret_cast<bf16*>(slots[rank]);
  for (int i = 0; i < n; ++i) {
    p.peer_slot[i] = reinterpret_cast<const bf16*>(slots[i]);
    p.peer_ready[i] = reinterpret_cast<const unsigned long long*>(ready[i]);
  }
  p.my_ready = reinterpret_cast<unsigned long long*>(ready[rank]);
  p.ctr = reinterpret_cast<unsigned int*>(ctrs.data_ptr());
  p.chunk_done = reinterpret_cast<unsigned long long*>(ctrs.data_ptr()) + 1;
  p.C = reinterpret_cast<bf16*>(y.data_ptr());
  p.ldc = y.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const bf16*>(bias->data_ptr()) : nullptr;
  p.status = device_status(x_full_out.get_device());
  const int dev = x_full_out.get_device();
  const int grid = num_sms(dev);
  if (trace.has_value()) {
    TORCH_CHECK(trace->numel() >= grid * 8 && trace->scalar_type() == at::kLong, "ag_gemm: trace [grid, 8] int64");
    p.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr());
  }
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  TmaSlots& ts = tls_tma_slots();
  const bool wide = N > 128;
  make_tma_2d_bf16(&ts.m[0], x_full_out.data_ptr(), K, M, K, 64, 128);
  make_tma_2d_bf16(&ts.m[1], w.data_ptr(), w.size(1), w.size(0), w.stride(0), 64, b_mn ? 64 : (wide ? 256 : 128));
  make_tma_2d_bf16(&ts.m[2], x_local.data_ptr(), K, M / n, K, 64, 128);
  NTB_CUDA_CHECK(cudaMemsetAsync(ctrs.data_ptr(), 0, sizeof(int64_t) * (1 + n), stream));
  void* args[4] = {&ts.m[0], &ts.m[1], &ts.m[2], &p};
  const int threads = 192 + 32 * kAgCopyWarps;
  if (wide) {
    if (b_mn) fused_launch(ag_gemm_kernel<256, true>, grid, FusedCfg<256>::SMEM_BYTES, args, stream, threads);
    else fused_launch(ag_gemm_kernel<256, false>, grid, FusedCfg<256>::SMEM_BYTES, args, stream, threads);
  } else {
    if (b_mn) fused_launch(ag_gemm_kernel<128, true>, grid, FusedCfg<128>::SMEM_BYTES, args, stream, threads);
    else fused_launch(ag_gemm_kernel<128, false>, grid, FusedCfg<128>::SMEM_BYTES, args, stream, threads);
  }
}

// x: [n*T_local, K] local operand; out: [T_local, N]
// recv: int64 [n] device addresses of every rank's receive slot base for this epoch ([n][T_local][N] bf16)
// tctrs: int64 [n] device addresses of every rank's per-tile arrival counters for this epoch parity
//        (T_local/128 * ceil(N/128) u32 each, zero at rest)
// ctrs: int64 [>=1] local scratch (tile counter), zeroed here per call
void gemm_rs(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, const c10::optional<at::Tensor>& bias,
             bool b_mn, std::vector<int64_t> recv, std::vector<int64_t> tctrs, at::Tensor& ctrs, int64_t rank,
             int64_t epoch, const c10::optional<at::Tensor>& trace) {
  const int n = static_cast<int>(recv.size());
  TORCH_CHECK(n >= 1 && n <= kMaxRanks && static_cast<int>(tctrs.size()) == n, "gemm_rs: 1..8 ranks");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm_rs: bf16");
  TORCH_CHECK(x.is_contiguous() && w.stride(1) == 1 && out.is_contiguous(), "gemm_rs: layouts");
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(M % n == 0 && (M / n) % 128 == 0, "gemm_rs: rows per rank must be a multiple of 128");
  const int64_t N = b_mn ? w.size(1) : w.size(0);
  TORCH_CHECK((b_mn ? w.size(0) : w.size(1)) == K, "gemm_rs: K mismatch");
  TORCH_CHECK(out.size(0) == M / n && out.size(1) == N, "gemm_rs: out");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "gemm_rs: K, N multiples of 8");
  TORCH_CHECK(ctrs.scalar_type() == at::kLong && ctrs.numel() >= 1 && ctrs.is_contiguous(), "gemm_rs: ctrs");
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
    p.peer_tctr[i] = reinterpret_cast<unsigned int*>(tctrs[i]);
  }
  p.my_tctr = reinterpret_cast<unsigned int*>(tctrs[rank]);
  p.my_recv = reinterpret_cast<const bf16*>(recv[rank]);
  p.ctr = reinterpret_cast<unsigned int*>(ctrs.data_ptr());
  p.out = reinterpret_cast<bf16*>(out.data_ptr());
  p.ldo = out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const bf16*>(bias->data_ptr()) : nullptr;
  p.status = device_status(x.get_device());
  const int dev = x.get_device();
  const int grid = num_sms(dev);
  if (trace.has_value()) {
    TORCH_CHECK(trace->numel() >= grid * 8 && trace->scalar_type() == at::kLong, "gemm_rs: trace [grid, 8] int64");
    p.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr());
  }
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  TmaSlots& ts = tls_tma_slots();
  const bool wide = N > 128;
  make_tma_2d_bf16(&ts.m[0], x.data_ptr(), K, M, x.stride(0), 64, 128);
  make_tma_2d_bf16(&ts.m[1], w.data_ptr(), w.size(1), w.size(0), w.stride(0), 64, b_mn ? 64 : (wide ? 256 : 128));
  NTB_CUDA_CHECK(cudaMemsetAsync(ctrs.data_ptr(), 0, sizeof(int64_t), stream));
  void* args[3] = {&ts.m[0], &ts.m[1], &p};
  if (wide) {
    if (b_mn) fused_launch(gemm_rs_kernel<256, true>, grid, FusedCfg<256>::SMEM_BYTES, args, stream, 224);
    else fused_launch(gemm_rs_kernel<256, false>, grid, FusedCfg<256>::SMEM_BYTES, args, stream, 224);
  } else {
    if (b_mn) fused_launch(gemm_rs_kernel<128, true>, grid, FusedCfg<128>::SMEM_BYTES, args, stream, 224);
    else fused_launch(gemm_rs_kernel<128, false>, grid, FusedCfg<128>::SMEM_BYTES, args, stream, 224);
  }
}


// x: [n*T_local, K]; out: [T_local, N] with N a multiple of the tile width.
// parts: int64 [n] every rank's partial slot base for this epoch parity ([n][T_local][N] bf16)
// rdy: int64 [n] address of rank r's ready words for source = this rank; my_rdy: this rank's
//      ready words [n][tpc_stride] (u64 epochs, monotonic)
// acc: fp32 [>= T_local * N] zero at rest; acc_cnt: int32 [>= tiles per chunk] zero at rest
void gemm_rsp(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, const c10::optional<at::Tensor>& bias,
              bool b_mn, std::vector<int64_t> parts, std::vector<int64_t> rdy, int64_t my_rdy, int64_t tpc_stride,
              at::Tensor& acc, at::Tensor& acc_cnt, at::Tensor& ctrs, int64_t rank, int64_t epoch,
              const c10::optional<at::Tensor>& trace) {
  const int n = static_cast<int>(parts.size());
  TORCH_CHECK(n >= 1 && n <= kMaxRanks && static_cast<int>(rdy.size()) == n, "gemm_rsp: 1..8 ranks");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm_rsp: bf16");
  TORCH_CHECK(x.is_contiguous() && w.stride(1) == 1 && out.is_contiguous(), "gemm_rsp: layouts");
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(M % n == 0 && (M / n) % 128 == 0, "gemm_rsp: rows per rank must be a multiple of 128");
  const int64_t N = b_mn ? w.size(1) : w.size(0);
  TORCH_CHECK((b_mn ? w.size(0) : w.size(1)) == K, "gemm_rsp: K mismatch");
  TORCH_CHECK(out.size(0) == M / n && out.size(1) == N, "gemm_rsp: out");
  TORCH_CHECK(K % 8 == 0, "gemm_rsp: K multiple of 8");
  const bool wide = N % 256 == 0;
  TORCH_CHECK(N % 128 == 0, "gemm_rsp: N must be a multiple of 128");
  const int BN = wide ? 256 : 128;
  const int64_t tpc = (M / n / 128) * (N / BN);
  TORCH_CHECK(tpc <= tpc_stride, "gemm_rsp: tiles per chunk exceed the ready-word stride");
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.numel() >= (M / n) * N && acc.is_contiguous(), "gemm_rsp: acc");
  TORCH_CHECK(acc_cnt.scalar_type() == at::kInt && acc_cnt.numel() >= tpc, "gemm_rsp: acc_cnt");
  TORCH_CHECK(ctrs.scalar_type() == at::kLong && ctrs.numel() >= 1 && ctrs.is_contiguous(), "gemm_rsp: ctrs");
  RspParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.T_local = static_cast<int>(M / n);
  p.n = n;
  p.rank = static_cast<int>(rank);
  p.tpc_stride = static_cast<int>(tpc_stride);
  p.epoch = static_cast<unsigned long long>(epoch);
  for (int i = 0; i < n; ++i) {
    TORCH_CHECK(parts[i] % 16 == 0, "gemm_rsp: 16-byte aligned partial slots");
    p.peer_part[i] = reinterpret_cast<const bf16*>(parts[i]);
    p.peer_rdy[i] = reinterpret_cast<unsigned long long*>(rdy[i]);
  }
  p.my_part = reinterpret_cast<bf16*>(parts[rank]);
  p.my_rdy = reinterpret_cast<const unsigned long long*>(my_rdy);
  p.acc = acc.data_ptr<float>();
  p.acc_cnt = reinterpret_cast<unsigned int*>(acc_cnt.data_ptr());
  p.ctr = reinterpret_cast<unsigned int*>(ctrs.data_ptr());
  p.out = reinterpret_cast<bf16*>(out.data_ptr());
  p.ldo = out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const bf16*>(bias->data_ptr()) : nullptr;
  const int dev = x.get_device();
  p.status = device_status(dev);
  const int grid = num_sms(dev);
  if (trace.has_value()) {
    TORCH_CHECK(trace->numel() >= grid * 8 && trace->scalar_type() == at::kLong, "gemm_rsp: trace [grid, 8] int64");
    p.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr());
  }
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  TmaSlots& ts = tls_tma_slots();
  make_tma_2d_bf16(&ts.m[0], x.data_ptr(), K, M, x.stride(0), 64, 128);
  make_tma_2d_bf16(&ts.m[1], w.data_ptr(), w.size(1), w.size(0), w.stride(0), 64, b_mn ? 64 : BN);
  NTB_CUDA_CHECK(cudaMemsetAsync(ctrs.data_ptr(), 0, sizeof(int64_t), stream));  // tile and pull-item counters
  void* args[3] = {&ts.m[0], &ts.m[1], &p};
  const int threads = 224 + 32 * kRspPullWarps;
  if (wide) {
    if (b_mn) fused_launch(gemm_rsp_kernel<256, true>, grid, FusedCfg<256>::SMEM_BYTES, args, stream, threads);
    else fused_launch(gemm_rsp_kernel<256, false>, grid, FusedCfg<256>::SMEM_BYTES, args, stream, threads);
  } else {
    if (b_mn) fused_launch(gemm_rsp_kernel<128, true>, grid, FusedCfg<128>::SMEM_BYTES, args, stream, threads);
    else fused_launch(gemm_rsp_kernel<128, false>, grid, FusedCfg<128>::SMEM_BYTES, args, stream, threads);
  }
}

// ================================================================== pull reduce-scatter
// out[T_local, N] = sum_r part_r[rank * T_local : (rank + 1) * T_local, :] (+ bias), part_r being rank r's
// full GEMM partial in its symmetric slot. Called after every rank published its partial; each
// thread issues its n peer loads before it adds them (fixed rank order, so every rank reduces
// its rows the same way), 16 bytes per load.
struct RsPullParams {
  const bf16* part[kMaxRanks];  // rank r's partial, already offset to this rank's first row
  bf16* out;
  const bf16* bias;
  long rows, N, ld_part, ld_out;
  int n;
  // Optional wait (flags != nullptr): before reading, every CTA waits (bounded) until each of the n
  // epoch words flags[0..n) - written by the ranks' publishing GEMMs - reaches `epoch`.
  const unsigned long long* flags;
  unsigned long long epoch;
  int* status;
};

__global__ void __launch_bounds__(256) rs_pull_kernel(const __grid_constant__ RsPullParams p) {
  if (p.flags != nullptr) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
      bool good = true;
      for (int s = 0; s < p.n && good; ++s)
        good = spin_until([&] { return ld_acquire_sys_u64(p.flags + s) >= p.epoch; }, p.status, kStatusTimeoutPeer);
      ok = good ? 1 : 0;
    }
    __syncthreads();  // the acquiring thread's view of the peers' partials, for the whole CTA
    if (!ok) return;
  }
  const long cpr = p.N / 8;  // 16-byte chunks per row
  const long total = p.rows * cpr;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long r = i / cpr, c = (i - r * cpr) * 8;
    uint4 v[kMaxRanks];
#pragma unroll
    for (int s = 0; s < kMaxRanks; ++s)
      if (s < p.n) v[s] = *reinterpret_cast<const uint4*>(p.part[s] + r * p.ld_part + c);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < kMaxRanks; ++s)
      if (s < p.n) {
        acc[0] += bf16_lo(v[s].x); acc[1] += bf16_hi(v[s].x); acc[2] += bf16_lo(v[s].y); acc[3] += bf16_hi(v[s].y);
        acc[4] += bf16_lo(v[s].z); acc[5] += bf16_hi(v[s].z); acc[6] += bf16_lo(v[s].w); acc[7] += bf16_hi(v[s].w);
      }
    if (p.bias != nullptr) {
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u] += __bfloat162float(p.bias[c + u]);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(p.out + r * p.ld_out + c) = o;
  }
}

// parts: int64 [n] device addresses of every rank's partial [n * T_local, N] (row pitch N)
void rs_pull(std::vector<int64_t> parts, at::Tensor& out, const c10::optional<at::Tensor>& bias, int64_t rank,
             int64_t flags_ptr, int64_t epoch) {
  const int n = static_cast<int>(parts.size());
  TORCH_CHECK(n >= 1 && n <= kMaxRanks && rank >= 0 && rank < n, "rs_pull: 1..8 ranks");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.is_contiguous(),
              "rs_pull: out bf16 [T_local, N]");
  const int64_t rows = out.size(0), N = out.size(1);
  TORCH_CHECK(N % 8 == 0, "rs_pull: N multiple of 8");
  if (bias.has_value())
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N && bias->is_contiguous(), "rs_pull: bias");
  RsPullParams p{};
  for (int i = 0; i < n; ++i) {
    TORCH_CHECK(parts[i] % 16 == 0, "rs_pull: 16-byte aligned partials");
    p.part[i] = reinterpret_cast<const bf16*>(parts[i]) + rank * rows * N;
  }
  p.out = reinterpret_cast<bf16*>(out.data_ptr());
  p.bias = bias.has_value() ? reinterpret_cast<const bf16*>(bias->data_ptr()) : nullptr;
  p.rows = rows;
  p.N = N;
  p.ld_part = N;
  p.ld_out = N;
  p.n = n;
  const int dev = out.get_device();
  p.flags = reinterpret_cast<const unsigned long long*>(flags_ptr);
  p.epoch = static_cast<unsigned long long>(epoch);
  p.status = device_status(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  const long chunks = rows * (N / 8);
  const int grid = static_cast<int>(std::max<long>(1, std::min<long>((chunks + 255) / 256, num_sms(dev) * 8L)));
  rs_pull_kernel<<<grid, 256, 0, stream>>>(p);
  NTB_LAUNCH_CHECK(1);
}

// ================================================================== bounded flag wait
// One thread waits until *flag >= expect (acquire, system scope) for at most
// limit_ns; on expiry it records kStatusTimeoutPeer in the device status word
// and returns. This is the wait the fused kernels use on peer flags, exposed
// on its own so the host-side timeout handling can be exercised with a flag
// that nothing sets.
__global__ void wait_flag_kernel(const unsigned int* flag, unsigned int expect, unsigned long long limit_ns,
                                 int* status) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys_u32(flag) < expect) {
    if (globaltimer_ns() - t0 > limit_ns) {
      set_status(status, kStatusTimeoutPeer);
      return;
    }
  }
}

void wait_flag(const at::Tensor& flag, int64_t expect, int64_t limit_ns) {
  TORCH_CHECK(flag.is_cuda() && flag.scalar_type() == at::kInt && flag.numel() >= 1, "wait_flag: int32 CUDA flag");
  TORCH_CHECK(limit_ns > 0 && limit_ns <= 10'000'000'000LL, "wait_flag: limit in (0, 10 s]");
  const int dev = flag.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev);
  wait_flag_kernel<<<1, 32, 0, stream>>>(reinterpret_cast<const unsigned int*>(flag.data_ptr()),
                                         static_cast<unsigned int>(expect),
                                         static_cast<unsigned long long>(limit_ns), device_status(dev));
  NTB_LAUNCH_CHECK(1);
}

}  // namespace ntb
