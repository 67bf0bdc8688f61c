"""Symmetric-memory communicator for the fused tensor-parallel kernels.

Each rank of a tensor-parallel group allocates one device buffer of the same
layout (``cudaMalloc`` + CUDA IPC handle, exchanged once through the process
group) and opens every peer's buffer, so the fused kernels address peer
memory directly over NVLink:

    [0, 4 KiB)          control words: AG ready epoch (u64 @0); pull reduce-scatter
                        "partial written" epochs (u64 [8 sources] @512)
    RS tile counters x2 per-tile arrival counters (u32, one per 128 x 128 output
                        tile of this rank's chunk) per epoch parity; zero at rest
    AG slots  x2        this rank's activation shard [T_local, K] per epoch parity
    RS recv   x2        partial tiles from every source rank [n][T_local][N] (fused push
                        reduce-scatter), or this rank's whole GEMM partial [n*T_local][N]
                        that the peers read (pull and progressive-pull reduce-scatter); all
                        kinds share one epoch counter, so a slot is reused only two
                        reduce-scatters later
    RS ready            progressive pull: per (source rank, output tile of this rank's chunk)
                        the epoch at which the source published the tile (u64, monotonic)
Every section after the control words is followed by a 256-byte canary
(``check_canaries``, parallel/region.py).

Only this rank's own buffer is ever viewed as a torch tensor; peer pointers
are handed to the fused kernels only.
"""
from __future__ import annotations

import os
import warnings

import torch
import torch.distributed as dist

from ..ops._ext import ext
from . import comm
from .fused import register_communicator
from .region import RegionLayout

_CTRL = 4096


class TPCommunicator:
    def __init__(self, group, *, max_local_rows: int, max_k: int, max_rs_n: int, device=None):
        self.group = group
        self.n = comm.group_size(group)
        self.rank = comm.group_rank(group)
        if self.n > 8:
            raise ValueError("TPCommunicator supports up to 8 ranks (one node)")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self.max_local_rows = max_local_rows
        self.max_k = max_k
        self.max_rs_n = max_rs_n
        self.ag_slot_bytes = max_local_rows * max_k * 2
        self.rs_slot_bytes = self.n * max_local_rows * max_rs_n * 2
        n_tiles = (max_local_rows // 128) * ((max_rs_n + 127) // 128)
        self.tctr_bytes = (n_tiles * 4 + 4095) // 4096 * 4096
        lay = RegionLayout(_CTRL)
        self.tctr_offs = [lay.add(f"rs_tile_counters{i}", self.tctr_bytes) for i in range(2)]
        self.ag_offs = [lay.add(f"ag_slot{i}", self.ag_slot_bytes) for i in range(2)]
        self.rs_offs = [lay.add(f"rs_slot{i}", self.rs_slot_bytes) for i in range(2)]
        self.tpc_stride = n_tiles  # tiles of one chunk at the narrowest (128-wide) tile
        self.rdy_off = lay.add("rs_ready", self.n * self.tpc_stride * 8)
        self.layout = lay
        total = lay.total
        C = ext()
        self.local_ptr, handle = C.symm_alloc(total)
        handles = [None] * self.n
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs = []
        self._opened = []
        for i, h in enumerate(handles):
            if i == self.rank:
                self.ptrs.append(self.local_ptr)
            else:
                p = C.symm_open(h)
                self.ptrs.append(p)
                self._opened.append(p)
        # Local scratch of the fused kernels (tile/piece counters, per-chunk copy counts); zeroed per call.
        self.ctrs = torch.zeros(1 + self.n, dtype=torch.int64, device=self.device)
        self.pub_ctr = torch.zeros(1, dtype=torch.int32, device=self.device)  # GEMM arrival count, zero at rest
        self.ag_epoch = 0
        self.rs_epoch = 0
        self.closed = False
        lay.fill(C, self.local_ptr, self.device.index)
        C.symm_local_view(self.local_ptr, self.rdy_off, [self.n * self.tpc_stride], torch.int64,
                          self.device.index).zero_()
        # Progressive pull: local fp32 sum of the peers' tiles of this rank's chunk, and the number of
        # sources added per tile; both zero at rest (the own-chunk epilogue re-zeroes what it used).
        self.rsp_acc = torch.zeros(max_local_rows * max_rs_n, dtype=torch.float32, device=self.device)
        self.rsp_cnt = torch.zeros(self.tpc_stride, dtype=torch.int32, device=self.device)
        # Optional int64 [num_sms, 8] tensor: per-CTA %globaltimer stamps of the last fused call.
        self.trace = None
        dist.barrier(group=group)

    # ------------------------------------------------------------------ layout helpers
    def _ready_ptrs(self):
        return [p + 0 for p in self.ptrs]

    def _ag_slot_ptrs(self, parity: int):
        return [p + self.ag_offs[parity] for p in self.ptrs]

    def _rs_recv_ptrs(self, parity: int):
        return [p + self.rs_offs[parity] for p in self.ptrs]

    def _rs_tctr_ptrs(self, parity: int):
        return [p + self.tctr_offs[parity] for p in self.ptrs]

    def check_canaries(self) -> list[str]:
        """Sections of this rank's region whose trailing canary was overwritten (synchronises)."""
        return self.layout.check(ext(), self.local_ptr, self.device.index)

    def supports(self, x: torch.Tensor, w: torch.Tensor) -> bool:
        return (not self.closed and x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
                and x.dim() == 2 and x.shape[-1] % 8 == 0)

    def all_gather_gemm_fits(self, x_shard: torch.Tensor, weight: torch.Tensor, b_mn: bool = False) -> bool:
        T_local, K = x_shard.shape
        return T_local <= self.max_local_rows and K <= self.max_k and T_local % 128 == 0

    def gemm_reduce_scatter_fits(self, x: torch.Tensor, weight: torch.Tensor, b_mn: bool = False) -> bool:
        T = x.shape[0]
        N = weight.shape[1] if b_mn else weight.shape[0]
        T_local = T // self.n
        return T % self.n == 0 and T_local <= self.max_local_rows and N <= self.max_rs_n and T_local % 128 == 0

    # ------------------------------------------------------------------ fused ops
    def all_gather_gemm(self, x_shard: torch.Tensor, weight: torch.Tensor, bias=None, b_mn: bool = False):
        T_local, K = x_shard.shape
        N = weight.shape[1] if b_mn else weight.shape[0]
        if T_local > self.max_local_rows or K > self.max_k or T_local % 128 != 0:
            return None
        self.ag_epoch += 1
        parity = self.ag_epoch & 1
        x_shard = x_shard.contiguous()
        full = torch.empty(self.n * T_local, K, dtype=torch.bfloat16, device=x_shard.device)
        y = torch.empty(self.n * T_local, N, dtype=torch.bfloat16, device=x_shard.device)
        ext().ag_gemm(x_shard, full, weight, y, bias, b_mn, self._ag_slot_ptrs(parity), self._ready_ptrs(),
                      self.ctrs, self.rank, self.ag_epoch, trace=self.trace)
        return y, full

    def gemm_reduce_scatter_pull(self, x: torch.Tensor, weight: torch.Tensor, b_mn: bool = False, bias=None):
        """GEMM into this rank's symmetric slot whose last CTA publishes the epoch to every rank, then one
        pull kernel that waits for every rank's epoch and sums this rank's rows of every partial (peer
        loads, fixed rank order). Two launches; no separate signal or wait kernel."""
        T, K = x.shape
        N = weight.shape[1] if b_mn else weight.shape[0]
        T_local = T // self.n
        if T % self.n or T_local > self.max_local_rows or N > self.max_rs_n or N % 8:
            return None
        self.rs_epoch += 1
        parity = self.rs_epoch & 1
        C = ext()
        dev = x.device.index
        part = C.symm_local_view(self.local_ptr, self.rs_offs[parity], [T, N], torch.bfloat16, dev)
        C.gemm_bf16_publish(x.contiguous(), weight, part, b_mn, [p + 512 + self.rank * 8 for p in self.ptrs],
                            self.rs_epoch, self.pub_ctr)
        out = torch.empty(T_local, N, dtype=torch.bfloat16, device=x.device)
        C.rs_pull(self._rs_recv_ptrs(parity), out, bias, self.rank, self.local_ptr + 512, self.rs_epoch)
        return out

    def gemm_reduce_scatter_overlap(self, x: torch.Tensor, weight: torch.Tensor, b_mn: bool = False, bias=None):
        """One kernel: GEMM tiles stored locally and released per tile; two warps per CTA pull this
        rank's chunk from every source as the sources finish it and sum it in fp32 while the GEMM
        runs; the own-chunk epilogue adds that sum (``csrc/tp_fused.cu``, gemm_rsp_kernel)."""
        T, K = x.shape
        N = weight.shape[1] if b_mn else weight.shape[0]
        T_local = T // self.n
        if T % self.n or T_local > self.max_local_rows or N > self.max_rs_n or T_local % 128 or N % 128:
            return None
        self.rs_epoch += 1
        parity = self.rs_epoch & 1
        out = torch.empty(T_local, N, dtype=torch.bfloat16, device=x.device)
        ext().gemm_rsp(x.contiguous(), weight, out, bias, b_mn, self._rs_recv_ptrs(parity),
                       [p + self.rdy_off + self.rank * self.tpc_stride * 8 for p in self.ptrs],
                       self.local_ptr + self.rdy_off, self.tpc_stride, self.rsp_acc, self.rsp_cnt, self.ctrs,
                       self.rank, self.rs_epoch, trace=self.trace)
        return out

    def gemm_reduce_scatter(self, x: torch.Tensor, weight: torch.Tensor, b_mn: bool = False, bias=None):
        T, K = x.shape
        N = weight.shape[1] if b_mn else weight.shape[0]
        T_local = T // self.n
        if T % self.n or T_local > self.max_local_rows or N > self.max_rs_n or T_local % 128 != 0:
            return None
        self.rs_epoch += 1
        parity = self.rs_epoch & 1
        out = torch.empty(T_local, N, dtype=torch.bfloat16, device=x.device)
        ext().gemm_rs(x, weight, out, bias, b_mn, self._rs_recv_ptrs(parity), self._rs_tctr_ptrs(parity),
                      self.ctrs, self.rank, self.rs_epoch, trace=self.trace)
        return out

    def close(self):
        if self.closed:
            return
        self.closed = True
        torch.cuda.synchronize()
        C = ext()
        for p in self._opened:
            C.symm_close(p)
        C.symm_free(self.local_ptr)


class _FusedAdapter:
    """Fused-dispatch interface over a TPCommunicator.

    Shapes the communicator cannot take fall back to NCCL + GEMM. With
    ``autotune`` (default, ``NTB_FUSED_AUTOTUNE=0`` disables it) the first
    call of every (op, shape, layout) times the candidates on the device
    (CUDA events, a few repetitions, max over the group so every rank takes
    the same decision) and later calls use the fastest: for the all-gather,
    the fused kernel vs NCCL + GEMM; for the reduce-scatter, the fused
    push-epilogue kernel, GEMM + the pull reduce-scatter kernel, and GEMM +
    NCCL (the push epilogue wins at two ranks, its remote stores limit it at
    eight).
    """

    REPS = 10
    REF = "nccl"       # the NCCL + GEMM candidate is the numerical reference of the others
    REL_TOL = 2e-2     # bf16 outputs; the candidates differ only in summation order

    def __init__(self, c: TPCommunicator, autotune: bool = True):
        self.c = c
        self.autotune = autotune
        self.choice: dict = {}  # key -> "fused" | "nccl"
        self.timings: dict = {}
        self.rel_err: dict = {}  # key -> {candidate: max over ranks of |y - y_nccl| / |y_nccl|}
        self.rejected: dict = {}  # key -> candidates dropped for disagreeing with NCCL + GEMM
        # NTB_FUSED_STRICT=1: a disagreeing candidate raises instead of being dropped (tests).
        self.strict = os.environ.get("NTB_FUSED_STRICT", "0") == "1"

    def supports(self, x, w):
        return self.c.supports(x, w)

    # ------------------------------------------------------------------ baseline paths
    def _ag_nccl(self, x_shard, weight, bias, b_mn):
        from ..ops.linear import gemm

        full = comm.all_gather_dim0(x_shard, self.c.group)
        return gemm(full, weight, bias=bias, b_mn=b_mn), full

    def _rs_nccl(self, x, weight, b_mn):
        from ..ops.linear import gemm

        return comm.reduce_scatter_dim0(gemm(x, weight, b_mn=b_mn), self.c.group)

    def _time(self, fn) -> float:
        fn()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(self.REPS):
            fn()
        e.record()
        e.synchronize()
        return s.elapsed_time(e) / self.REPS

    def _decide(self, key, candidates: dict) -> str:
        """Name of the fastest candidate (first one when autotune is off); timed on the device, max over
        the group, so every rank takes the same decision.

        Before timing, every candidate's output on this call's operands is compared with the NCCL +
        GEMM candidate's (relative L2 error, max over the group, recorded in ``rel_err``); a fused
        kernel that disagrees beyond ``REL_TOL`` is dropped for that shape with a warning (recorded
        in ``rejected``), or raises with NTB_FUSED_STRICT=1. This is the multi-GPU correctness check
        of the fused kernels that runs inside every multi-GPU job."""
        ch = self.choice.get(key)
        if ch is not None:
            return ch
        names = list(candidates)
        if not self.autotune:
            self.choice[key] = names[0]
            return names[0]
        order = [self.REF] + [k for k in names if k != self.REF] if self.REF in names else names
        ref, errs = None, {}
        for k in order:
            out = candidates[k]()
            y = (out[0] if isinstance(out, tuple) else out).detach().float()
            if k == self.REF:
                ref = y.clone()
            elif ref is not None:
                errs[k] = float(((y - ref).norm() / ref.norm().clamp_min(1e-30)).item())
        err_names = list(errs)
        vals = [self._time(candidates[k]) for k in names] + [errs[k] for k in err_names]
        t = torch.tensor(vals, dtype=torch.float64, device=self.c.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.c.group)
        got = [float(v) for v in t]
        times, err_max = got[:len(names)], dict(zip(err_names, got[len(names):]))
        self.rel_err[key] = {k: float(f"{v:.3e}") for k, v in err_max.items()}
        bad = {k: v for k, v in err_max.items() if not v <= self.REL_TOL}
        if bad:
            if self.strict:
                raise RuntimeError(f"fused kernel output differs from NCCL + GEMM for {key}: relative error "
                                   f"{bad} > {self.REL_TOL}")
            # Not used for this shape (every rank sees the same reduced errors, so all drop it).
            warnings.warn(f"fused candidates {sorted(bad)} disagree with NCCL + GEMM for {key} "
                          f"(relative error {bad}); using the others")
            self.rejected[key] = bad
        ok = [i for i, k in enumerate(names) if k not in bad]
        ch = names[min(ok, key=lambda i: times[i])]
        self.choice[key] = ch
        self.timings[key] = dict(zip(names, (round(v, 4) for v in times)))
        return ch

    # ------------------------------------------------------------------ fused ops
    def all_gather_gemm(self, x_shard, weight, bias, b_mn=False):
        key = ("ag", tuple(x_shard.shape), tuple(weight.shape), b_mn, bias is not None)
        if self.c.all_gather_gemm_fits(x_shard, weight, b_mn):
            ch = self._decide(key, {"fused": lambda: self.c.all_gather_gemm(x_shard, weight, bias, b_mn=b_mn),
                                    "nccl": lambda: self._ag_nccl(x_shard, weight, bias, b_mn)})
            if ch == "fused":
                return self.c.all_gather_gemm(x_shard, weight, bias, b_mn=b_mn)
        return self._ag_nccl(x_shard, weight, bias, b_mn)

    def gemm_reduce_scatter(self, x, weight, b_mn=False):
        key = ("rs", tuple(x.shape), tuple(weight.shape), b_mn)
        if self.c.gemm_reduce_scatter_fits(x, weight, b_mn):
            cands = {"fused": lambda: self.c.gemm_reduce_scatter(x, weight, b_mn=b_mn),
                     "pull": lambda: self.c.gemm_reduce_scatter_pull(x, weight, b_mn=b_mn),
                     "nccl": lambda: self._rs_nccl(x, weight, b_mn)}
            N = weight.shape[1] if b_mn else weight.shape[0]
            if N % 128 == 0 and os.environ.get("NTB_FUSED_RS_OVERLAP", "0") == "1":
                cands["overlap"] = lambda: self.c.gemm_reduce_scatter_overlap(x, weight, b_mn=b_mn)
            ch = self._decide(key, cands)
            if ch == "fused":
                return self.c.gemm_reduce_scatter(x, weight, b_mn=b_mn)
            if ch == "pull":
                return self.c.gemm_reduce_scatter_pull(x, weight, b_mn=b_mn)
            if ch == "overlap":
                return self.c.gemm_reduce_scatter_overlap(x, weight, b_mn=b_mn)
        return self._rs_nccl(x, weight, b_mn)

    def all_gather(self, x_shard):
        return comm.all_gather_dim0(x_shard, self.c.group)

    def close(self):
        self.c.close()


def maybe_attach_communicator(group, *, max_local_rows: int = 4096, max_k: int = 4096, max_rs_n: int = 4096):
    """Register a fused-kernel communicator on a single-node NCCL group of CUDA ranks.

    Disabled with NTB_FUSED_TP=0 (the NCCL + GEMM baseline then runs).
    """
    if os.environ.get("NTB_FUSED_TP", "1") == "0":
        return None
    if not (torch.cuda.is_available() and dist.is_initialized() and comm.group_size(group) > 1):
        return None
    if dist.get_backend(group) != "nccl":
        return None
    c = TPCommunicator(group, max_local_rows=max_local_rows, max_k=max_k, max_rs_n=max_rs_n)
    a = _FusedAdapter(c, autotune=os.environ.get("NTB_FUSED_AUTOTUNE", "1") != "0")
    register_communicator(group, a)
    return a
