"""Row-window sharding across the GPUs of one box.

Windows are independent and write disjoint output rows, so the path shards
with no data-path collective: rank r owns a contiguous window range
[lo_r, hi_r) cut at equal cost prefix sums, holds the Q / O rows of that
range (its slab) and a replica of K and V.  The only collective is the
optional all-gather of O, for callers that need the full output on every
rank.

Cost of a window = its active blocks + WINDOW_COST: every block moves a K and
a V tile (64*d bytes per head), every window reads a Q tile and writes an O
tile (32*d + 64*d bytes per head), i.e. 1.5 blocks' worth.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import numpy as np

WINDOW_COST = 1.5


def partition_windows(window_offsets, world_size: int, window_cost: float = WINDOW_COST) -> List[Tuple[int, int]]:
    """Contiguous [lo, hi) window ranges, one per rank, of near-equal cost."""
    off = np.asarray(window_offsets, dtype=np.int64)
    nrw = off.shape[0] - 1
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    cost = np.diff(off).astype(np.float64) + window_cost
    prefix = np.concatenate([[0.0], np.cumsum(cost)])
    total = prefix[-1]
    cuts = [0]
    for r in range(1, world_size):
        c = int(np.searchsorted(prefix, total * r / world_size, side="left"))
        cuts.append(min(max(c, cuts[-1]), nrw))
    cuts.append(nrw)
    return [(cuts[r], cuts[r + 1]) for r in range(world_size)]


def slab_rows(lo: int, hi: int, num_nodes: int) -> Tuple[int, int]:
    """Node rows [r0, r1) covered by windows [lo, hi)."""
    return min(16 * lo, num_nodes), min(16 * hi, num_nodes)


def rank_order(global_order, lo: int, hi: int):
    """The global balanced order restricted to [lo, hi), order preserved
    (still descending by block count).  Works on numpy arrays and torch
    tensors alike."""
    keep = (global_order >= lo) & (global_order < hi)
    return global_order[keep]


def gather_rows(slab, slabs: Sequence[Tuple[int, int]], group=None):
    """All-gather per-rank row slabs (torch tensors, first dim = rows) into
    the full tensor on every rank.  Slabs may differ in size: each rank pads
    to the largest slab, one all_gather moves them, and the padding is
    dropped.  Every rank makes the same collective call."""
    import torch
    import torch.distributed as dist

    sizes = [r1 - r0 for r0, r1 in slabs]
    m = max(sizes) if sizes else 0
    if slab.shape[0] != sizes[dist.get_rank(group)]:
        raise ValueError("slab rows disagree with the partition")
    padded = torch.zeros((m,) + tuple(slab.shape[1:]), dtype=slab.dtype, device=slab.device)
    padded[: slab.shape[0]] = slab
    bufs = [torch.empty_like(padded) for _ in sizes]
    dist.all_gather(bufs, padded, group=group)
    return torch.cat([b[:s] for b, s in zip(bufs, sizes)], dim=0)


def sub_ranges(window_offsets, lo: int, hi: int, parts: int, window_cost: float = WINDOW_COST):
    """[lo, hi) cut into `parts` contiguous window ranges of near-equal cost
    (some may be empty)."""
    off = np.asarray(window_offsets, dtype=np.int64)[lo:hi + 1]
    local = partition_windows(off - off[0], parts, window_cost) if hi > lo else [(0, 0)] * parts
    return [(lo + a, lo + b) for a, b in local]


class OverlappedGather:
    """All-gather of O rows, one sub-slab at a time, overlapped with the
    computation of the next sub-slab.

    Every rank cuts its window range into the same number of sub-slabs
    (`sub_slabs`, cost-balanced), so every rank makes the same collective
    calls in the same order.  After the caller has enqueued the computation
    of sub-slab j on the current stream, `send(j, o_slab)` makes a side
    stream wait for it, pads this rank's rows of sub-slab j to the largest
    rank's, all-gathers them and copies every rank's rows into the full O.
    `finish()` makes the current stream wait for the side stream and returns
    the full O ([num_nodes, ...] on every rank).  On CPU tensors (gloo) the
    same calls run synchronously."""

    def __init__(self, window_offsets, parts, rank: int, num_nodes: int, row_shape, dtype, device,
                 sub_slabs: int = 4, group=None):
        import torch

        self.rank, self.group, self.num_nodes = rank, group, num_nodes
        self.parts = list(parts)
        self.subs = [sub_ranges(window_offsets, lo, hi, sub_slabs) for lo, hi in self.parts]
        self.rows = [[slab_rows(a, b, num_nodes) for a, b in s] for s in self.subs]
        self.row_shape = tuple(row_shape)
        self.device = torch.device(device)
        self.full = torch.empty((num_nodes,) + self.row_shape, dtype=dtype, device=self.device)
        self.cuda = self.device.type == "cuda"
        self.stream = torch.cuda.Stream(self.device) if self.cuda else None
        self.sub_slabs = sub_slabs
        m = [max(r[j][1] - r[j][0] for r in self.rows) for j in range(sub_slabs)]
        self.max_rows = m
        self.stage = [torch.zeros((mj,) + self.row_shape, dtype=dtype, device=self.device) for mj in m]
        self.recv = [torch.empty((len(self.parts) * mj,) + self.row_shape, dtype=dtype, device=self.device)
                     for mj in m]

    def my_sub_ranges(self):
        return self.subs[self.rank]

    def start(self):
        """Called before the first sub-slab of a step (nothing to do here)."""

    def output_slab(self, shape, dtype):
        """Where the forward writes this rank's O rows."""
        import torch

        return torch.empty(shape, dtype=dtype, device=self.device)

    def _exchange(self, j: int, o_slab):
        import torch.distributed as dist

        mj = self.max_rows[j]
        if mj == 0:
            return
        r0 = slab_rows(*self.parts[self.rank], self.num_nodes)[0]
        a, b = self.rows[self.rank][j]
        if b > a:
            self.stage[j][: b - a].copy_(o_slab[a - r0:b - r0])
        views = [self.recv[j][q * mj:(q + 1) * mj] for q in range(len(self.parts))]
        dist.all_gather(views, self.stage[j], group=self.group)
        for q, (qa, qb) in enumerate(self.rows_of(j)):
            if qb > qa:
                self.full[qa:qb].copy_(views[q][: qb - qa])

    def rows_of(self, j: int):
        return [r[j] for r in self.rows]

    def send(self, j: int, o_slab):
        import torch

        if not self.cuda:
            self._exchange(j, o_slab)
            return
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            self._exchange(j, o_slab)
            o_slab.record_stream(self.stream)

    def finish(self):
        import torch

        if self.cuda:
            torch.cuda.current_stream(self.device).wait_stream(self.stream)
        return self.full


def sharded_forward_allgather(Q_slab, K, V, fmt, global_order, parts, rank: int, window_offsets=None,
                              sub_slabs: int = 4, out_dtype=None, block_hints=None, plans=None, group=None,
                              gather: Optional["OverlappedGather"] = None):
    """This rank's windows of O computed in `sub_slabs` launches, each
    followed by an all-gather of its rows that overlaps the next launch;
    returns the full O on every rank (bit-identical to a 1-GPU run).

    Q_slab: this rank's Q rows (slab_rows of parts[rank]); K, V replicated;
    global_order: the balanced order of all windows; plans: optional list of
    per-sub-slab plans (make_plan over each sub-slab's order)."""
    import torch
    from . import api as F

    if window_offsets is None:
        window_offsets = fmt.window_offsets.cpu().numpy()
    dtype = out_dtype or torch.float32
    q3 = Q_slab if Q_slab.dim() == 3 else Q_slab.unsqueeze(1)
    og = gather or OverlappedGather(window_offsets, parts, rank, fmt.num_nodes, q3.shape[1:], dtype, Q_slab.device,
                                    sub_slabs, group)
    r0, _ = slab_rows(*parts[rank], fmt.num_nodes)
    o_slab = og.output_slab(q3.shape, dtype)
    og.start()
    for j, (a, b) in enumerate(og.my_sub_ranges()):
        ra, rb = slab_rows(a, b, fmt.num_nodes)
        if rb > ra:
            order_j = rank_order(global_order, a, b).contiguous()
            F.fused3s_forward(q3[ra - r0:rb - r0], K, V, fmt, order=order_j, out=o_slab[ra - r0:rb - r0],
                              q_window_base=a, block_hints=block_hints,
                              plan=None if plans is None else plans[j])
        og.send(j, o_slab)
    return og.finish()


class _DeviceBuffer:
    """A raw device allocation seen by torch (zero-copy) as uint8[nbytes]."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerGather:
    """All-gather of O rows by the copy engines over NVLink, overlapped with
    the fused kernel.

    Every rank allocates its full O in an IPC-exportable buffer
    (f3s_peer_alloc) and maps every other rank's (f3s_peer_open); the forward
    writes this rank's rows in place (`output_slab`).  After the
    computation of sub-slab j is enqueued, `send(j, o_slab)` makes a side
    stream wait for it and copies this rank's rows of sub-slab j into every
    other rank's full O (f3s_peer_copy: cudaMemcpyAsync, a copy engine, no SMs --
    so it runs beside a kernel that holds every SM, where a collective kernel
    would wait for one).  Two stream-ordered handshakes (a one-element NCCL
    all-reduce on the side stream) bracket a step: `start()` keeps peers from
    writing into this rank's full O before its earlier work on it is done,
    and `finish()` tells every rank that all copies into its buffer are
    complete, then makes the current stream wait.  Same interface as
    OverlappedGather; `close()` unmaps and frees (collective)."""

    def __init__(self, window_offsets, parts, rank: int, num_nodes: int, row_shape, dtype, device,
                 sub_slabs: int = 4, group=None):
        import ctypes
        import torch
        import torch.distributed as dist
        from . import _lib

        self.lib = _lib.load()
        self.rank, self.group, self.num_nodes = rank, group, num_nodes
        self.parts = list(parts)
        self.subs = [sub_ranges(window_offsets, lo, hi, sub_slabs) for lo, hi in self.parts]
        self.rows = [[slab_rows(a, b, num_nodes) for a, b in s] for s in self.subs]
        self.device = torch.device(device)
        self.row_shape = tuple(row_shape)
        elem = torch.empty(0, dtype=dtype).element_size()
        self.row_bytes = int(np.prod(self.row_shape)) * elem
        nbytes = max(num_nodes * self.row_bytes, 1)
        with torch.cuda.device(self.device):
            ptr = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(_lib.F3S_IPC_HANDLE_BYTES)
            _lib.check(self.lib.f3s_peer_alloc(nbytes, ctypes.byref(ptr), handle), "f3s_peer_alloc")
            self.ptr = ptr.value
            handles = [None] * len(self.parts)
            dist.all_gather_object(handles, handle.raw, group=group)
            self.peer_ptrs = []
            for q, h in enumerate(handles):
                if q == rank:
                    self.peer_ptrs.append(self.ptr)
                    continue
                p = ctypes.c_void_p()
                _lib.check(self.lib.f3s_peer_open(ctypes.create_string_buffer(h, len(h)), ctypes.byref(p)),
                           "f3s_peer_open")
                self.peer_ptrs.append(p.value)
            raw = torch.as_tensor(_DeviceBuffer(self.ptr, nbytes), device=self.device)
            self.full = raw[: num_nodes * self.row_bytes].view(dtype).view((num_nodes,) + self.row_shape)
            self.stream = torch.cuda.Stream(self.device)
            self.flag = torch.zeros(1, dtype=torch.int32, device=self.device)

    def my_sub_ranges(self):
        return self.subs[self.rank]

    def output_slab(self, shape, dtype):
        """This rank's rows of the full O: the forward writes them in place."""
        r0, r1 = slab_rows(*self.parts[self.rank], self.num_nodes)
        if self.full.dtype != dtype or tuple(shape) != (r1 - r0,) + self.row_shape:
            raise ValueError("output slab shape / dtype disagree with the gather buffer")
        return self.full[r0:r1]

    def _handshake(self):
        import torch.distributed as dist

        dist.all_reduce(self.flag, group=self.group)

    def start(self):
        import torch

        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self._handshake()

    def send(self, j: int, o_slab):
        import torch

        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        r0 = slab_rows(*self.parts[self.rank], self.num_nodes)[0]
        a, b = self.rows[self.rank][j]
        if b > a:
            src = o_slab.data_ptr() + (a - r0) * self.row_bytes
            sptr = self.stream.cuda_stream
            for q, dst in enumerate(self.peer_ptrs):
                if dst + a * self.row_bytes == src:
                    continue  # written in place by the forward
                _lib_check(self.lib.f3s_peer_copy(dst + a * self.row_bytes, src, (b - a) * self.row_bytes, sptr))
        # o_slab is this gatherer's own buffer (output_slab), alive as long as it is

    def finish(self):
        import torch

        with torch.cuda.stream(self.stream):
            self._handshake()
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        return self.full

    def close(self):
        """Collective: every rank unmaps the others' buffers, then frees its own."""
        import torch
        import torch.distributed as dist

        if self.ptr is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for q, p in enumerate(self.peer_ptrs):
            if q != self.rank:
                self.lib.f3s_peer_close(p)
        dist.barrier(group=self.group)
        self.full = None
        self.lib.f3s_peer_free(self.ptr)
        self.ptr = None


def _lib_check(status: int):
    from . import _lib

    _lib.check(status, "f3s_peer_copy")
