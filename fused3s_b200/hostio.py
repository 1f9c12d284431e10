"""The fused forward with its inputs and its output in host memory.

The reference's harness copies Q, K, V to the device before every launch and
O back after it (tests/test_fused_3s_v2.cu:97-120, 133-135).  HostForward is
that call for this engine, with the copies overlapped with the work:

  * K and V go first (every window may read any row of them).  On one GPU
    the whole of K and V is uploaded; with K / V sharded over the ranks of a
    process group (`kv_share=(rank, world)`), each rank uploads only its
    1/world share of the rows from its own host memory and an NCCL
    all-gather over NVLink assembles the replica on every rank, so the
    host-to-device traffic per rank falls as 1/world;
  * the caller's windows are cut into `sub_slabs` cost-balanced row ranges:
    sub-slab j's Q rows are uploaded on a copy stream, its forward (with its
    own work plan) waits only for them, and its O rows go back to the host on
    a second copy stream while the next sub-slab computes.

Host buffers must be pinned (page-locked) for the copies to be asynchronous:
`pinned_empty` allocates such a buffer of exactly the requested size
(cudaHostRegister on an ordinary allocation; torch's pinned allocator rounds
large requests up to a power of two).
"""
from __future__ import annotations

import weakref
from typing import Optional, Sequence, Tuple

import numpy as np
import torch

from . import api as F
from . import shard


def pinned_empty(shape, dtype: torch.dtype) -> torch.Tensor:
    """A host tensor whose memory is page-locked for the GPU (registered with
    cudaHostRegister; unregistered when the tensor is freed)."""
    t = torch.empty(shape, dtype=dtype)
    nbytes = t.numel() * t.element_size()
    if nbytes == 0:
        return t
    rt = torch.cuda.cudart()
    err = rt.cudaHostRegister(t.data_ptr(), nbytes, 0)
    if int(err) != 0:
        raise RuntimeError(f"cudaHostRegister of {nbytes} bytes failed ({int(err)})")
    ptr = t.data_ptr()
    weakref.finalize(t, rt.cudaHostUnregister, ptr)
    return t


def kv_share_rows(num_nodes: int, world: int) -> Tuple[int, Sequence[Tuple[int, int]]]:
    """Rows of K / V each rank contributes when K / V are sharded over
    `world` ranks: equal shares of whole block columns (`share_rows` each,
    a multiple of 16), the last ones cut at num_nodes.  Returns (share_rows,
    [(r0, r1) per rank])."""
    nrw = (num_nodes + 15) // 16
    share = 16 * (-(-nrw // world)) if world > 0 else 0
    rows = [(min(r * share, num_nodes), min((r + 1) * share, num_nodes)) for r in range(world)]
    return share, rows


class HostForward:
    """O = fused3s_forward(Q, K, V) for a window range, from and to host
    memory, with the copies overlapped (see the module docstring).

    fmt: the graph's format (on this device); order: the balanced order of
    all windows (default: computed); window_range: the windows [lo, hi) this
    caller computes (default all; a rank's slab from shard.partition_windows);
    kv_share: (rank, world) when every rank holds only its share of K / V on
    the host (kv_share_rows) and a process group is initialised, else None;
    block_hints: optional per-block L2 hints; out_dtype: element type of O.

    run(hQ, hK, hV, hO): hQ = the range's Q rows [q_rows, H, d] fp16, hK / hV
    = this caller's K / V rows (all of them, or its share), hO = [q_rows, H, d]
    of out_dtype; all pinned host tensors.  Enqueued on the current stream
    (which waits for the copy streams at the end); returns hO.
    buffers: optional (dQ, dK, dV, dO) device tensors to use instead of
    allocating them (their contents are overwritten every run)."""

    def __init__(self, fmt: F.BlockSparseFormat, heads: int, head_dim: int, order: Optional[torch.Tensor] = None,
                 window_range: Optional[Tuple[int, int]] = None, kv_share: Optional[Tuple[int, int]] = None,
                 block_hints: Optional[torch.Tensor] = None, sub_slabs: int = 4,
                 out_dtype: torch.dtype = torch.float32, group=None, buffers=None):
        self.fmt, self.heads, self.head_dim = fmt, heads, head_dim
        self.device = fmt.window_offsets.device
        N = fmt.num_nodes
        if order is None:
            order = F.generate_balanced_window_order(fmt)
        lo, hi = window_range if window_range is not None else (0, fmt.num_row_windows)
        self.lo, self.hi = lo, hi
        self.r0, self.r1 = shard.slab_rows(lo, hi, N)
        off_h = fmt.window_offsets.cpu().numpy()
        self.subs = [(a, b) for a, b in shard.sub_ranges(off_h, lo, hi, max(1, sub_slabs))]
        self.plans = []
        for a, b in self.subs:
            o = shard.rank_order(order, a, b).contiguous()
            self.plans.append(F.make_plan(fmt, heads, head_dim, order=o) if o.numel() else None)
        self.hints = block_hints
        self.out_dtype = out_dtype
        self.group = group
        self.kv_share = kv_share
        if kv_share is not None:
            rank, world = kv_share
            self.share_rows, self.share_ranges = kv_share_rows(N, world)
            kv_rows = world * self.share_rows
        else:
            rank, world = 0, 1
            self.share_rows, self.share_ranges = N, [(0, N)]
            kv_rows = N
        self.rank, self.world = rank, world
        shape = (heads, head_dim)
        dev = self.device
        if buffers is not None:
            # the caller's device buffers (Q slab, K, V with kv_rows rows, O
            # slab): reused instead of allocated -- at C5's size one set of
            # device buffers is half the GPU's memory
            self.dQ, self.dK, self.dV, self.dO = buffers
            if (tuple(self.dQ.shape) != (self.r1 - self.r0,) + shape or self.dK.shape[0] < max(kv_rows, 1)
                    or self.dV.shape[0] < max(kv_rows, 1) or tuple(self.dO.shape) != (self.r1 - self.r0,) + shape
                    or self.dO.dtype != out_dtype):
                raise ValueError("buffers do not fit the window range / K / V rows / O type")
        else:
            self.dQ = torch.empty((self.r1 - self.r0,) + shape, dtype=torch.float16, device=dev)
            self.dK = torch.empty((max(kv_rows, 1),) + shape, dtype=torch.float16, device=dev)
            self.dV = torch.empty((max(kv_rows, 1),) + shape, dtype=torch.float16, device=dev)
            self.dO = torch.empty((self.r1 - self.r0,) + shape, dtype=out_dtype, device=dev)
        self.s_in = torch.cuda.Stream(dev)
        self.s_out = torch.cuda.Stream(dev)

    @property
    def h2d_bytes(self) -> int:
        """Host-to-device bytes of one run (this caller's)."""
        a, b = self.share_ranges[self.rank]
        row = self.heads * self.head_dim * 2
        return (self.r1 - self.r0) * row + 2 * (b - a) * row

    @property
    def d2h_bytes(self) -> int:
        return (self.r1 - self.r0) * self.heads * self.head_dim * self.dO.element_size()

    def run(self, hQ: torch.Tensor, hK: torch.Tensor, hV: torch.Tensor, hO: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        N = self.fmt.num_nodes
        a, b = self.share_ranges[self.rank]
        if hK.shape[0] != b - a or hV.shape[0] != b - a:
            raise ValueError(f"K / V host rows {hK.shape[0]} / {hV.shape[0]}: this caller holds rows [{a}, {b})")
        if hQ.shape[0] != self.r1 - self.r0 or hO.shape[0] != self.r1 - self.r0:
            raise ValueError("Q / O host rows disagree with the window range")
        cur = torch.cuda.current_stream(self.device)
        # earlier work on the device buffers (the previous run) comes first
        self.s_in.wait_stream(cur)
        self.s_out.wait_stream(cur)
        base = self.rank * self.share_rows
        with torch.cuda.stream(self.s_in):
            if b > a:
                self.dK[base:base + (b - a)].copy_(hK, non_blocking=True)
                self.dV[base:base + (b - a)].copy_(hV, non_blocking=True)
        kv_ready = torch.cuda.Event()
        kv_ready.record(self.s_in)
        q_ready = []
        with torch.cuda.stream(self.s_in):
            for sa, sb in self.subs:
                ra, rb = shard.slab_rows(sa, sb, N)
                if rb > ra:
                    self.dQ[ra - self.r0:rb - self.r0].copy_(hQ[ra - self.r0:rb - self.r0], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.s_in)
                q_ready.append(ev)
        cur.wait_event(kv_ready)
        if self.world > 1:
            # every rank's share -> the replica on every rank (in place, NVLink)
            for t in (self.dK, self.dV):
                dist.all_gather_into_tensor(t, t[base:base + self.share_rows], group=self.group)
        K, V = self.dK[:N], self.dV[:N]
        for j, (sa, sb) in enumerate(self.subs):
            ra, rb = shard.slab_rows(sa, sb, N)
            if rb <= ra:
                continue
            cur.wait_event(q_ready[j])
            F.fused3s_forward(self.dQ[ra - self.r0:rb - self.r0], K, V, self.fmt,
                              out=self.dO[ra - self.r0:rb - self.r0], q_window_base=sa, block_hints=self.hints,
                              plan=self.plans[j])
            done = torch.cuda.Event()
            done.record(cur)
            self.s_out.wait_event(done)
            with torch.cuda.stream(self.s_out):
                hO[ra - self.r0:rb - self.r0].copy_(self.dO[ra - self.r0:rb - self.r0], non_blocking=True)
        cur.wait_stream(self.s_out)
        cur.wait_stream(self.s_in)
        return hO
