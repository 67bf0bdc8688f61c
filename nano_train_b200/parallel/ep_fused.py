"""Fused expert-parallel MoE dispatch / combine over NVLink peer memory.

The reference exchanges MoE tokens with ``all_to_all_single`` after a host
synchronisation on the per-rank counts (src/models/moe.py:640-1146: count
exchange + ``.tolist()``, payload / metadata / weight all-to-alls, capacity
``topk`` per expert, reverse all-to-all, ``index_add_``). Here the exchange is
kernels writing and reading peer memory directly (csrc/moe_ep.cu), and
nothing waits on the host:

forward   plan_send (device sorts) -> ep_dispatch: payload rows, optionally
          e4m3 with 1x128 scales, stored straight into each destination's slab
          -> bounded wait for every source -> plan_receive (capacity selection
          by weight per expert, device sorts) -> ep_gather into the
          zero-padded expert-grouped layout -> grouped SwiGLU GEMMs writing
          the expert outputs into the workspace -> ep_pull: each source reads
          its tokens' K expert rows from the peers and sums w_k * y_k.
backward  ep_combine_bwd: each expert rank reads dOut rows of its sources
          and scales them by the routing weight -> grouped GEMM backward
          writes dX into the workspace -> ep_pull with unit weights sums the K
          expert-input gradients of every token.

``plan_send`` and ``plan_receive`` are plain torch and run on the CPU too:
the gloo tests drive them through an in-process emulation of the kernels
(``emulate_exchange``) against the unfused all-to-all module.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from . import comm
from .region import RegionLayout

FLAG_DISPATCH, FLAG_Y, FLAG_DOUT, FLAG_DX = range(4)
MAX_RANKS = 8
MAX_TOPK = 8
SEG = 128


# ---------------------------------------------------------------------------- planning (pure torch)
@dataclass
class SendPlan:
    tok: torch.Tensor          # int32 [T*K] token of each destination-sorted assignment
    dest: torch.Tensor         # int32 [T*K] destination rank
    slot: torch.Tensor         # int32 [T*K] row in this source's block of the destination slab
    lexp: torch.Tensor         # int32 [T*K] expert index local to the destination
    kslot: torch.Tensor        # int32 [T*K] top-k slot
    w: torch.Tensor            # fp32  [T*K] routing weight (detached)
    send_counts: torch.Tensor  # int32 [n] rows per destination
    dest_tk: torch.Tensor      # int32 [T*K] destination of assignment (t, k), token order
    slot_tk: torch.Tensor      # int32 [T*K] slab row of assignment (t, k)


def plan_send(topk_idx: torch.Tensor, topk_w: torch.Tensor, experts_per_rank: int, n: int) -> SendPlan:
    """Sort this rank's (token, k) assignments by global expert (hence by destination rank)."""
    T, K = topk_idx.shape
    flat_e = topk_idx.reshape(-1).long()
    order = torch.argsort(flat_e, stable=True)
    de = flat_e[order]
    dest = torch.div(de, experts_per_rank, rounding_mode="floor")
    send_counts = torch.bincount(dest, minlength=n)
    starts = torch.cumsum(send_counts, 0) - send_counts
    slot = torch.arange(order.numel(), device=order.device) - starts[dest]
    dest_tk = torch.empty_like(dest)
    dest_tk[order] = dest
    slot_tk = torch.empty_like(slot)
    slot_tk[order] = slot
    i32 = torch.int32
    return SendPlan(tok=(order // K).to(i32), dest=dest.to(i32), slot=slot.to(i32),
                    lexp=(de - dest * experts_per_rank).to(i32), kslot=(order % K).to(i32),
                    w=topk_w.detach().reshape(-1)[order].float().contiguous(), send_counts=send_counts.to(i32),
                    dest_tk=dest_tk.to(i32), slot_tk=slot_tk.to(i32))


def _desc_float_key(bits: torch.Tensor) -> torch.Tensor:
    """int32 float bit patterns -> int64 in [0, 2^32) ascending in DEScending float order."""
    b = bits.long() & 0xFFFFFFFF
    neg = b >= 0x80000000
    asc = torch.where(neg, (~b) & 0xFFFFFFFF, b | 0x80000000)  # monotone in the float value
    return 0xFFFFFFFF - asc


@dataclass
class RecvPlan:
    offsets: torch.Tensor      # int32 [E_local + 1] padded row offsets of the grouped layout
    rows: int                  # host bound on the grouped rows (multiple of 128)
    row_src: torch.Tensor      # int32 [rows] source rank of each grouped row, -1 = padding
    row_slot: torch.Tensor     # int32 [rows] slab row inside the source's block
    row_tok: torch.Tensor      # int32 [rows] token index on the source
    row_w: torch.Tensor        # fp32  [rows] routing weight
    rowmap: torch.Tensor       # int32 [n * P] grouped row of each slab row, -1 = dropped / empty
    kept_counts: torch.Tensor  # int64 [E_local]
    stats: torch.Tensor        # fp32 [2] (dropped, received)


def receive_keys(recv_counts: torch.Tensor, meta: torch.Tensor, experts_per_rank: int, top_k: int):
    """Total order of the received rows (ascending = kept first), as ep_recv_keys computes it:
    local expert (empty rows last), weight descending, source rank, the source's t * K + k."""
    n, P = meta.shape[0], meta.shape[1]
    epr = experts_per_rank
    valid = torch.arange(P, device=meta.device)[None, :] < recv_counts.clamp(0, P).view(n, 1)
    le = torch.where(valid, meta[..., 0].clamp(0, epr - 1), torch.full_like(meta[..., 0], epr)).reshape(-1).long()
    src = torch.arange(n, device=meta.device).view(n, 1).expand(n, P).reshape(-1)
    flat = (meta[..., 1].long() * top_k + meta[..., 3].long()).reshape(-1) & 0xFFFFF
    key = (le << 55) | (_desc_float_key(meta[..., 2].reshape(-1)) << 23) | (src << 20) | flat
    return key, valid, le


def plan_receive(recv_counts: torch.Tensor, meta: torch.Tensor, experts_per_rank: int, capacity: torch.Tensor,
                 rows_bound: int, top_k: int) -> RecvPlan:
    """Capacity selection and the expert-grouped layout of the received rows (PyTorch form of
    ep_recv_keys + sort + ep_recv_layout, used by the CPU tests).

    ``meta`` int32 [n, P, 4] holds {local expert, token, weight bits, k} per slab
    row; rows p >= recv_counts[s] of source s are empty. Each expert keeps its
    ``capacity`` highest-weight assignments, ties in arrival order of the unfused
    module (source rank, then the source's assignments in token order) whatever
    order the rows landed in the slab.
    """
    n, P = meta.shape[0], meta.shape[1]
    epr = experts_per_rank
    dev = meta.device
    key, valid, le = receive_keys(recv_counts, meta, epr, top_k)
    o = torch.argsort(key)
    le_s = le[o]
    counts_all = torch.bincount(le_s, minlength=epr + 1)
    starts = torch.cumsum(counts_all, 0) - counts_all
    rank_in = torch.arange(o.numel(), device=dev) - starts[le_s]
    keep = (le_s < epr) & (rank_in < capacity)
    kept_counts = torch.minimum(counts_all[:epr], capacity)
    padded = (kept_counts + (SEG - 1)) // SEG * SEG
    offsets = torch.zeros(epr + 1, dtype=torch.int32, device=dev)
    offsets[1:] = torch.cumsum(padded, 0).to(torch.int32)
    rows = (rows_bound + SEG - 1) // SEG * SEG
    pos = offsets[le_s.clamp(max=epr - 1)].long() + rank_in
    dump = torch.full_like(pos, rows)  # one scratch row past the end takes the non-kept entries
    tgt = torch.where(keep, pos, dump)
    src = (o // P).to(torch.int32)
    slot = (o % P).to(torch.int32)
    minus1 = torch.full_like(src, -1)
    row_src = torch.full((rows + 1,), -1, dtype=torch.int32, device=dev)
    row_src.scatter_(0, tgt, torch.where(keep, src, minus1))
    row_slot = torch.zeros(rows + 1, dtype=torch.int32, device=dev).scatter_(0, tgt, slot)
    meta_flat = meta.reshape(-1, 4)
    row_tok = torch.zeros(rows + 1, dtype=torch.int32, device=dev).scatter_(0, tgt, meta_flat[o, 1])
    row_w = torch.zeros(rows + 1, dtype=torch.float32, device=dev).scatter_(
        0, tgt, meta_flat[o, 2].contiguous().view(torch.float32))
    rowmap = torch.empty(n * P, dtype=torch.int32, device=dev)
    rowmap.scatter_(0, o, torch.where(keep, pos, torch.full_like(pos, -1)).to(torch.int32))
    received = valid.sum()
    stats = torch.stack([(received - keep.sum()).float(), received.float()])
    return RecvPlan(offsets=offsets, rows=rows, row_src=row_src[:rows].contiguous(),
                    row_slot=row_slot[:rows].contiguous(), row_tok=row_tok[:rows].contiguous(),
                    row_w=row_w[:rows].contiguous(), rowmap=rowmap, kept_counts=kept_counts, stats=stats)


def capacity_tensor(t_all: torch.Tensor, capacity_factor: float, top_k: int, num_experts: int,
                    host_cap: int) -> torch.Tensor:
    """max(ceil(cf * T_all * K / E), 1) on the device (same float64 arithmetic as the host formula),
    clamped to the host bound the buffers were sized for."""
    cap = torch.ceil(capacity_factor * t_all.double() * top_k / float(num_experts)).clamp(min=1).long()
    return torch.clamp(cap, max=host_cap)


def rows_bound(n: int, P: int, experts_per_rank: int, host_cap: int) -> int:
    return min(n * P, experts_per_rank * host_cap) + experts_per_rank * (SEG - 1)


# ---------------------------------------------------------------------------- CPU emulation of the kernels
def emulate_exchange(tokens: list, plans: list, experts_per_rank: int, P: int):
    """What ep_dispatch leaves in every destination: (recv_counts [n], meta [n, P, 4], payload [n, P, H]).

    ``tokens[s]`` / ``plans[s]`` are source s's tokens and SendPlan (CPU tensors).
    """
    n = len(plans)
    H = tokens[0].shape[1]
    out = []
    for d in range(n):
        counts = torch.zeros(n, dtype=torch.int32)
        meta = torch.zeros(n, P, 4, dtype=torch.int32)
        payload = torch.zeros(n, P, H, dtype=tokens[0].dtype)
        for s in range(n):
            sp = plans[s]
            sel = (sp.dest == d).nonzero().flatten()
            counts[s] = sel.numel()
            slots = sp.slot[sel].long()
            meta[s, slots, 0] = sp.lexp[sel]
            meta[s, slots, 1] = sp.tok[sel]
            meta[s, slots, 2] = sp.w[sel].view(torch.int32)
            meta[s, slots, 3] = sp.kslot[sel]
            payload[s, slots] = tokens[s][sp.tok[sel].long()]
        out.append((counts, meta, payload))
    return out


def emulate_gather(payload: torch.Tensor, rp: RecvPlan) -> torch.Tensor:
    """ep_gather: grouped rows from the slab ([n, P, H]), zero for padding."""
    n, P, H = payload.shape
    flat = payload.reshape(n * P, H)
    idx = (rp.row_src.clamp(min=0).long() * P + rp.row_slot.long())
    x = flat[idx]
    return torch.where((rp.row_src >= 0).view(-1, 1), x, torch.zeros_like(x))


def emulate_pull(T: int, K: int, sp: SendPlan, rowmaps: list, ys: list, w_tk: Optional[torch.Tensor], me: int,
                 P: int) -> torch.Tensor:
    """ep_pull on the CPU: out[t] = sum_k w[t, k] * y_dest[rowmap_dest[me * P + slot]] (fp32 sum)."""
    H = ys[0].shape[1]
    out = torch.zeros(T, H, dtype=torch.float32)
    for a in range(T * K):
        d = int(sp.dest_tk[a])
        pos = int(rowmaps[d][me * P + int(sp.slot_tk[a])])
        if pos >= 0:
            w = 1.0 if w_tk is None else float(w_tk[a])
            out[a // K] += w * ys[d][pos].float()
    return out


# ---------------------------------------------------------------------------- symmetric workspace
def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


class EPWorkspace:
    """One symmetric buffer per rank of an expert-parallel group (CUDA IPC).

    Layout (offsets identical on every rank):
        ctrl     flags u64 [4 kinds][8 sources] @0, info int32 [8 sources][4] @256
        meta     int4  [n][P]        per received row {local expert, token, weight bits, k}
        payload  bf16 or e4m3 [n][P][H]  received rows, block s written by source s
        pscale   fp32  [n][P][H/128]     (e4m3 payload)
        rowmap   int32 [n][P]        grouped row of each received row (-1 dropped)
        y        bf16  [R][H]        expert outputs (read by the sources)
        yq, ys   e4m3 [R][H], fp32 [R][H/128]  (e4m3 combine)
        dx       bf16  [R][H]        gradient of the expert inputs (read by the sources)
        dout     bf16  [T][H]        gradient of this rank's MoE output (read by the expert ranks)
    P = max_tokens * top_k rows per source, R = n * P + E_local * 128 rows.
    """

    def __init__(self, group, *, max_tokens: int, hidden: int, top_k: int, experts_per_rank: int,
                 fp8_payload: bool, device=None):
        from ..ops._ext import ext

        self.group = group
        self.n = comm.group_size(group)
        self.rank = comm.group_rank(group)
        if self.n > MAX_RANKS:
            raise ValueError("EPWorkspace supports up to 8 ranks (one node)")
        if top_k > MAX_TOPK:
            raise ValueError("fused expert-parallel path supports top_k <= 8")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self.T, self.H, self.K, self.epr = max_tokens, hidden, top_k, experts_per_rank
        self.fp8 = fp8_payload
        n, H = self.n, hidden
        self.P = P = max_tokens * top_k
        self.R = R = _align(n * P + experts_per_rank * SEG, SEG)
        pay_elem = 1 if fp8_payload else 2
        lay = RegionLayout(4096)
        self.off_meta = lay.add("meta", n * P * 16)
        self.off_payload = lay.add("payload", n * P * H * pay_elem)
        self.off_pscale = lay.add("pscale", n * P * (H // 128) * 4 if fp8_payload else 0)
        self.off_rowmap = lay.add("rowmap", n * P * 4)
        self.off_y = lay.add("y", R * H * 2)
        self.off_yq = lay.add("yq", R * H if fp8_payload else 0)
        self.off_ys = lay.add("ys", R * (H // 128) * 4 if fp8_payload else 0)
        self.off_dx = lay.add("dx", R * H * 2)
        self.off_dout = lay.add("dout", max_tokens * H * 2)
        self.layout = lay
        self.bytes = lay.total
        C = ext()
        self._C = C
        self.local, handle = C.symm_alloc(self.bytes)
        handles = [None] * n
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs, self._opened = [], []
        for i, h in enumerate(handles):
            if i == self.rank:
                self.ptrs.append(self.local)
            else:
                p = C.symm_open(h)
                self.ptrs.append(p)
                self._opened.append(p)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.ctr = torch.zeros(MAX_RANKS, dtype=torch.int32, device=self.device)
        lay.fill(C, self.local, self.device.index)
        self.epoch = [0, 0, 0, 0]
        self.closed = False
        dist.barrier(group=group)

    # -------------------------------------------------------------- views and pointers
    def _view(self, off: int, sizes, dtype):
        return self._C.symm_local_view(self.local, off, list(sizes), dtype, self.device.index)

    def info(self):
        return self._view(256, (self.n, 4), torch.int32)

    def meta(self):
        return self._view(self.off_meta, (self.n, self.P, 4), torch.int32)

    def rowmap(self):
        return self._view(self.off_rowmap, (self.n * self.P,), torch.int32)

    def y(self, rows: int):
        return self._view(self.off_y, (rows, self.H), torch.bfloat16)

    def dx(self, rows: int):
        return self._view(self.off_dx, (rows, self.H), torch.bfloat16)

    def dout(self, T: int):
        return self._view(self.off_dout, (T, self.H), torch.bfloat16)

    def _flag_ptrs(self, kind: int):
        """Each destination's flag word of `kind` for this source."""
        return [p + (kind * MAX_RANKS + self.rank) * 8 for p in self.ptrs]

    def _next(self, kind: int) -> int:
        self.epoch[kind] += 1
        return self.epoch[kind]

    def _signal_and_wait(self, kind: int):
        e = self._next(kind)
        self._C.ep_signal(self._flag_ptrs(kind), e, self.device.index)
        self._C.ep_wait(self.local + kind * MAX_RANKS * 8, self.n, e, self.device.index)

    # -------------------------------------------------------------- steps
    def dispatch(self, tokens: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor, *, stochastic: bool,
                 seed: int):
        """Sends every (token, k) row; returns (dest_tk, slot_tk) int32 [T*K]."""
        T, K = topk_idx.shape
        if T > self.T:
            raise ValueError(f"EPWorkspace sized for {self.T} tokens per rank, got {T}")
        me, P, H = self.rank, self.P, self.H
        pay_row = H * (1 if self.fp8 else 2)
        dest_tk = torch.empty(T * K, dtype=torch.int32, device=self.device)
        slot_tk = torch.empty(T * K, dtype=torch.int32, device=self.device)
        e = self._next(FLAG_DISPATCH)
        self._C.ep_dispatch(
            tokens, topk_idx, topk_w, dest_tk, slot_tk, self.ctr, self.epr,
            [p + self.off_payload + me * P * pay_row for p in self.ptrs],
            [p + self.off_pscale + me * P * (H // 128) * 4 for p in self.ptrs] if self.fp8 else [],
            [p + self.off_meta + me * P * 16 for p in self.ptrs],
            self._flag_ptrs(FLAG_DISPATCH),
            [p + 256 + me * 16 for p in self.ptrs],
            self.done, P, e, self.fp8, stochastic, seed)
        self._C.ep_wait(self.local + FLAG_DISPATCH * MAX_RANKS * 8, self.n, e, self.device.index)
        return dest_tk, slot_tk

    def plan(self, *, num_experts: int, capacity_factor: float, host_cap: int) -> RecvPlan:
        """Capacity selection + grouped layout of what arrived (ep_recv_keys, one sort, ep_recv_layout);
        writes the row map into the workspace for the sources' combine."""
        n, P, epr = self.n, self.P, self.epr
        dev = self.device
        counts = torch.zeros(epr, dtype=torch.int32, device=dev)
        keys = torch.empty(n * P, dtype=torch.int64, device=dev)
        self._C.ep_recv_keys(self.local + self.off_meta, self.local + 256, keys, counts, P, n, epr, self.K)
        skeys, order = torch.sort(keys)
        rows = (rows_bound(n, P, epr, host_cap) + SEG - 1) // SEG * SEG
        offsets = torch.empty(epr + 1, dtype=torch.int32, device=dev)
        row_src = torch.empty(rows, dtype=torch.int32, device=dev)
        row_slot = torch.empty(rows, dtype=torch.int32, device=dev)
        row_tok = torch.empty(rows, dtype=torch.int32, device=dev)
        row_w = torch.empty(rows, dtype=torch.float32, device=dev)
        stats = torch.empty(2, dtype=torch.float32, device=dev)
        self._C.ep_recv_layout(skeys, order, self.local + self.off_meta, self.local + 256, counts, offsets, row_src,
                               row_slot, row_tok, row_w, self.local + self.off_rowmap, stats, P, n, epr, self.K,
                               num_experts, float(capacity_factor), int(host_cap))
        return RecvPlan(offsets=offsets, rows=rows, row_src=row_src, row_slot=row_slot, row_tok=row_tok, row_w=row_w,
                        rowmap=None, kept_counts=torch.clamp(counts, max=host_cap), stats=stats)

    def gather(self, rp: RecvPlan) -> torch.Tensor:
        x = torch.empty(rp.rows, self.H, dtype=torch.bfloat16, device=self.device)
        self._C.ep_gather(x, rp.offsets[self.epr:], rp.row_src, rp.row_slot, self.local + self.off_payload,
                          self.local + self.off_pscale, self.P, self.n, self.fp8)
        return x

    def publish_y(self, rp: RecvPlan, *, stochastic: bool, seed: int):
        if self.fp8:
            self._C.ep_quant_rows(self.y(rp.rows), rp.offsets[self.epr:], self.local + self.off_yq,
                                  self.local + self.off_ys, stochastic, seed)
        self._signal_and_wait(FLAG_Y)

    def pull_combine(self, dest_tk: torch.Tensor, slot_tk: torch.Tensor, w_tk: torch.Tensor, T: int, save: bool):
        K = self.K
        out = torch.empty(T, self.H, dtype=torch.bfloat16, device=self.device)
        y_save = torch.empty(T * K, self.H, dtype=torch.bfloat16, device=self.device) if save else None
        pos = torch.empty(T * K, dtype=torch.int32, device=self.device)
        src = [p + (self.off_yq if self.fp8 else self.off_y) for p in self.ptrs]
        self._C.ep_pull(out, dest_tk, slot_tk, w_tk, None,
                        [p + self.off_rowmap + self.rank * self.P * 4 for p in self.ptrs], src,
                        [p + self.off_ys for p in self.ptrs] if self.fp8 else [], self.P, self.R, self.fp8,
                        y_save=y_save, pos_out=pos)
        return out, y_save, pos

    def combine_backward(self, dout: torch.Tensor, rp: RecvPlan, T: int) -> torch.Tensor:
        self.dout(T).copy_(dout)
        self._signal_and_wait(FLAG_DOUT)
        dy = torch.empty(rp.rows, self.H, dtype=torch.bfloat16, device=self.device)
        self._C.ep_combine_bwd(dy, rp.offsets[self.epr:], rp.row_src, rp.row_tok, rp.row_w,
                               [p + self.off_dout for p in self.ptrs], T)
        return dy

    def dispatch_backward(self, g_xpad: torch.Tensor, dest_tk: torch.Tensor, pos_tk: torch.Tensor, T: int):
        if g_xpad.data_ptr() != self.local + self.off_dx:
            self.dx(g_xpad.shape[0]).copy_(g_xpad)
        self._signal_and_wait(FLAG_DX)
        dx = torch.empty(T, self.H, dtype=torch.bfloat16, device=self.device)
        self._C.ep_pull(dx, dest_tk, dest_tk, None, pos_tk, [], [p + self.off_dx for p in self.ptrs], [],
                        self.P, self.R, False)
        return dx

    def check_canaries(self) -> list[str]:
        """Sections of this rank's region whose trailing canary was overwritten (synchronises)."""
        return self.layout.check(self._C, self.local, self.device.index)

    def close(self):
        if self.closed:
            return
        self.closed = True
        torch.cuda.synchronize()
        for p in self._opened:
            self._C.symm_close(p)
        self._C.symm_free(self.local)


_WORKSPACES: dict = {}


def workspaces() -> list:
    return list(_WORKSPACES.values())


def get_workspace(group, *, tokens: int, hidden: int, top_k: int, experts_per_rank: int, fp8: bool) -> EPWorkspace:
    """The group's workspace, created collectively on first use (every EP rank calls this at the same layer)."""
    key = (id(group), hidden, top_k, experts_per_rank, fp8)
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = EPWorkspace(group, max_tokens=tokens, hidden=hidden, top_k=top_k, experts_per_rank=experts_per_rank,
                         fp8_payload=fp8)
        _WORKSPACES[key] = ws
    return ws


def clear_workspaces():
    for ws in _WORKSPACES.values():
        ws.close()
    _WORKSPACES.clear()


def fused_ep_enabled(group) -> bool:
    if os.environ.get("NTB_FUSED_EP", "1") == "0":
        return False
    if not (torch.cuda.is_available() and dist.is_initialized()):
        return False
    n = comm.group_size(group)
    return comm.min_fused_ranks() <= n <= MAX_RANKS and dist.get_backend(group) == "nccl"


# ---------------------------------------------------------------------------- autograd
@dataclass
class _CallState:
    ws: EPWorkspace
    topk_idx: torch.Tensor
    topk_w: torch.Tensor
    T: int
    host_cap: int
    capacity_factor: float
    num_experts: int
    stochastic: bool
    dest_tk: Optional[torch.Tensor] = None
    slot_tk: Optional[torch.Tensor] = None
    rp: Optional[RecvPlan] = None
    pos_tk: Optional[torch.Tensor] = None


def _seed(stochastic: bool) -> int:
    return int(torch.randint(0, 2 ** 62, (1,)).item()) if stochastic else 0


class _EPDispatchFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, st: _CallState):
        ws = st.ws
        st.dest_tk, st.slot_tk = ws.dispatch(tokens.contiguous(), st.topk_idx, st.topk_w.detach().contiguous(),
                                             stochastic=st.stochastic, seed=_seed(st.stochastic))
        st.rp = ws.plan(num_experts=st.num_experts, capacity_factor=st.capacity_factor, host_cap=st.host_cap)
        ctx.st = st
        return ws.gather(st.rp)

    @staticmethod
    def backward(ctx, g):
        st = ctx.st
        return st.ws.dispatch_backward(g.contiguous(), st.dest_tk, st.pos_tk, st.T), None


class _EPCombineFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, w_tk, st: _CallState):
        ws = st.ws
        ws.publish_y(st.rp, stochastic=st.stochastic, seed=_seed(st.stochastic))
        out, y_save, pos = ws.pull_combine(st.dest_tk, st.slot_tk, w_tk.detach().contiguous(), st.T,
                                           save=ctx.needs_input_grad[1])
        st.pos_tk = pos
        ctx.st = st
        ctx.save_for_backward(y_save if y_save is not None else torch.empty(0))
        return out

    @staticmethod
    def backward(ctx, dout):
        st = ctx.st
        (y_save,) = ctx.saved_tensors
        dout = dout.contiguous().to(torch.bfloat16)
        dy = st.ws.combine_backward(dout, st.rp, st.T)
        dw = None
        if ctx.needs_input_grad[1]:
            T, K, H = st.T, st.ws.K, st.ws.H
            dw = torch.bmm(y_save.view(T, K, H), dout.view(T, H, 1)).view(-1).float()
        return dy, dw, None


def fused_ep_moe(tokens: torch.Tensor, topk_idx: torch.Tensor, topk_w: torch.Tensor, experts, stack_cache, *,
                 group, num_experts: int, capacity_factor: float, fp8_payload: bool, stochastic: bool):
    """Routed-expert output [T, H] of an expert-parallel MoE layer and (stats, kept_counts) device tensors."""
    from ..ops.grouped import GroupedBuffers, _GroupedSwiGLUFn, expert_operands, grouped_fp8_rounding

    n = comm.group_size(group)
    T, H = tokens.shape
    K = topk_idx.shape[1]
    epr = num_experts // n
    ws = get_workspace(group, tokens=T, hidden=H, top_k=K, experts_per_rank=epr, fp8=fp8_payload)
    host_cap = max(int(math.ceil(capacity_factor * (n * T) * K / float(num_experts))), 1)
    st = _CallState(ws=ws, topk_idx=topk_idx.contiguous(), topk_w=topk_w, T=T, host_cap=host_cap,
                    capacity_factor=capacity_factor, num_experts=num_experts, stochastic=stochastic)
    x_pad = _EPDispatchFn.apply(tokens, st)
    rp = st.rp
    fp8 = grouped_fp8_rounding(experts)
    w1, w2, codes = expert_operands(experts, stack_cache, fp8, x_pad.dtype)
    bufs = GroupedBuffers(y_out=ws.y(rp.rows), dx_out=ws.dx(rp.rows))
    y = _GroupedSwiGLUFn.apply(x_pad, rp.offsets, w1, w2, len(experts), bufs, fp8, codes,
                               *stack_cache.params(experts))
    out = _EPCombineFn.apply(y, topk_w.float().reshape(-1), st)
    return out.to(tokens.dtype), rp.stats, rp.kept_counts
