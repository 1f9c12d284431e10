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


def gather_rows(slab, slabs: Sequence[Tuple[int, int]], group=None, deadline_s: Optional[float] = None):
    """All-gather per-rank row slabs (torch tensors, first dim = rows) into
    the full tensor on every rank.  Slabs may differ in size: each rank pads
    to the largest slab, one all_gather moves them, and the padding is
    dropped.  Every rank makes the same collective call.  With deadline_s
    the host waits for the collective at most that long (guarded_wait): a
    rank that never joins makes the others raise CollectiveTimeout instead
    of hanging."""
    import torch
    import torch.distributed as dist

    sizes = [r1 - r0 for r0, r1 in slabs]
    m = max(sizes) if sizes else 0
    if slab.shape[0] != sizes[dist.get_rank(group)]:
        raise ValueError("slab rows disagree with the partition")
    padded = torch.zeros((m,) + tuple(slab.shape[1:]), dtype=slab.dtype, device=slab.device)
    padded[: slab.shape[0]] = slab
    bufs = [torch.empty_like(padded) for _ in sizes]
    with _nvtx("f3s_gather_rows", slab.device):
        if deadline_s is None:
            dist.all_gather(bufs, padded, group=group)
        else:
            guarded_wait(dist.all_gather(bufs, padded, group=group, async_op=True), deadline_s, group,
                         "all_gather of O")
    return torch.cat([b[:s] for b, s in zip(bufs, sizes)], dim=0)


class _nvtx:
    """NVTX range on CUDA devices (a no-op elsewhere)."""

    def __init__(self, name, device):
        self.name = name
        self.on = getattr(device, "type", None) == "cuda"

    def __enter__(self):
        if self.on:
            import torch
            torch.cuda.nvtx.range_push(self.name)
        return self

    def __exit__(self, *exc):
        if self.on:
            import torch
            torch.cuda.nvtx.range_pop()
        return False


# ----------------------------------------------------------------------------
# Failure detection across ranks (the host side; no GPU fault is involved)
# ----------------------------------------------------------------------------

class RankFailure(RuntimeError):
    """A rank did not reach a step within the deadline."""

    def __init__(self, missing, step, waited_s):
        self.missing, self.step, self.waited_s = list(missing), step, waited_s
        super().__init__(f"rank(s) {self.missing} did not reach step {step} within {waited_s:.1f}s")


class CollectiveTimeout(RuntimeError):
    """A collective did not complete within the deadline; the process group
    was aborted (every later collective on it fails at once)."""


def guarded_wait(work, deadline_s: float, group=None, what: str = "collective", poll_s: float = 0.005):
    """Wait for an async collective (a torch.distributed Work) for at most
    deadline_s seconds, polling its completion -- and, for NCCL, the
    communicator's asynchronous error, which a failed work raises from
    wait().  On expiry the process group is aborted (ProcessGroup.abort,
    i.e. ncclCommAbort for NCCL) so that nothing stays blocked on the dead
    peer, and CollectiveTimeout is raised."""
    import time
    import torch.distributed as dist

    t0 = time.monotonic()
    while True:
        if work.is_completed():
            try:
                work.wait()  # returns at once; raises the work's error, if any
            except Exception as err:
                raise CollectiveTimeout(f"{what} failed: {err}") from err
            return
        if time.monotonic() - t0 > deadline_s:
            pg = group if group is not None else dist.distributed_c10d._get_default_group()
            try:
                pg.abort()
            except Exception:  # a backend without abort: the group's own timeout ends the work
                pass
            raise CollectiveTimeout(f"{what} did not complete within {deadline_s:.1f}s; process group aborted")
        time.sleep(poll_s)


class Heartbeat:
    """Per-step liveness through a torch.distributed Store (the process
    group's, or any TCPStore).  Before step k every rank calls
    arrive(k) and then wait(k): wait returns once every rank arrived, or
    raises RankFailure naming the missing ranks after deadline_s -- so the
    surviving ranks learn of a rank that left between steps on the host,
    before they launch anything that would wait for it."""

    def __init__(self, store, rank: int, world: int, deadline_s: float = 30.0, prefix: str = "f3s/heartbeat"):
        self.store, self.rank, self.world = store, rank, world
        self.deadline_s, self.prefix = deadline_s, prefix

    def _key(self, step, rank):
        return f"{self.prefix}/{step}/{rank}"

    def arrive(self, step: int) -> None:
        self.store.set(self._key(step, self.rank), "1")

    def wait(self, step: int, poll_s: float = 0.01) -> None:
        import time
        t0 = time.monotonic()
        pending = [r for r in range(self.world) if r != self.rank]
        while pending:
            pending = [r for r in pending if not self.store.check([self._key(step, r)])]
            if not pending:
                return
            waited = time.monotonic() - t0
            if waited > self.deadline_s:
                raise RankFailure(pending, step, waited)
            time.sleep(poll_s)

    def step(self, step: int) -> None:
        self.arrive(step)
        self.wait(step)


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


# ----------------------------------------------------------------------------
# Ring-passed K / V slices (K / V larger than one GPU's memory)
# ----------------------------------------------------------------------------

def ring_slice_at(rank: int, step: int, world: int) -> int:
    """The K / V slice rank `rank` holds at ring step `step`: its own at step
    0, then its predecessor's, and so on (slice j starts on rank j)."""
    return (rank - step) % world


def ring_pass(rank: int, world: int, compute, send, handshake) -> None:
    """The ring schedule, independent of the transport.

    Two slots per rank.  At step s the rank holds slice ring_slice_at(rank, s)
    in slot s % 2 and calls compute(s, slice); meanwhile send(s) passes that
    slot to the next rank's slot (s + 1) % 2 (except at the last step).
    handshake(s) ends the step on every rank: afterwards the slot the rank
    received is complete, and the slot it computed on may be overwritten by
    its predecessor at step s + 1.  Every rank sees every slice exactly once."""
    for s in range(world):
        compute(s, ring_slice_at(rank, s, world))
        if s < world - 1:
            send(s)
        handshake(s)


class RingKV:
    """The fused forward of this rank's windows with K / V sharded over the
    ranks of a process group and passed around the ring, so no rank ever
    holds more than two slices of K / V (the reference reads all of K / V on
    one device, src/fused3s_v2.cu:152-165,216-225).

    Slice j of K / V is rank j's share: the rows of the block columns
    api.column_slices(num_nodes, world)[0][j] ... [j + 1].  The rank's
    windows [lo, hi) are cut at the slice boundaries into one work plan
    (make_sliced_plan); at ring step s the rank runs the plan's pieces for
    the slice it holds (f3s_forward_pieces, K / V pointing at that slice's
    rows), while the copy engine sends the slice on to the next rank over
    NVLink (CUDA IPC buffers, f3s_peer_copy: no SMs, so it overlaps the
    kernel); a one-element NCCL all-reduce ends each step.  After the last
    step the split windows are merged (f3s_plan_merge, in column order: the
    result is deterministic and independent of the world size's slice
    arrival order).

    run(Q_slab, K_share, V_share) -> O slab: Q_slab = this rank's Q rows
    (shard.slab_rows of its windows), K_share / V_share = this rank's slice
    rows [N, H, d][r0:r1] (slice_rows(rank))."""

    def __init__(self, fmt, heads: int, head_dim: int, window_range, rank: int, world: int, order=None,
                 block_hints=None, out_dtype=None, group=None):
        import ctypes
        import torch
        import torch.distributed as dist
        from . import _lib, api as F

        self.lib = _lib.load()
        self.fmt, self.heads, self.head_dim = fmt, heads, head_dim
        self.rank, self.world, self.group = rank, world, group
        self.device = fmt.window_offsets.device
        N = fmt.num_nodes
        self.lo, self.hi = window_range
        self.r0, self.r1 = slab_rows(self.lo, self.hi, N)
        self.cuts, self.slice_rows = F.column_slices(N, world)
        if order is None:
            order = F.generate_balanced_window_order(fmt)
        my_order = rank_order(order, self.lo, self.hi).contiguous()
        self.plan = F.make_sliced_plan(fmt, heads, head_dim, self.cuts, order=my_order)
        self.hints = block_hints
        self.out_dtype = out_dtype or torch.float32
        max_rows = max(b - a for a, b in self.slice_rows)
        self.row_bytes = heads * head_dim * 2
        self.slot_rows = max(max_rows, 1)
        slot_bytes = 2 * self.slot_rows * self.row_bytes  # K then V
        self.slot_bytes = slot_bytes
        with torch.cuda.device(self.device):
            self.ptrs, self.peer = [], []
            handles = []
            for _ in range(2):
                p = ctypes.c_void_p()
                h = ctypes.create_string_buffer(_lib.F3S_IPC_HANDLE_BYTES)
                _lib.check(self.lib.f3s_peer_alloc(slot_bytes, ctypes.byref(p), h), "f3s_peer_alloc")
                self.ptrs.append(p.value)
                handles.append(h.raw)
            every = [None] * world
            dist.all_gather_object(every, handles, group=group)
            nxt = (rank + 1) % world
            for hh in every[nxt]:  # the next rank's two slots, mapped here
                p = ctypes.c_void_p()
                _lib.check(self.lib.f3s_peer_open(ctypes.create_string_buffer(hh, len(hh)), ctypes.byref(p)),
                           "f3s_peer_open")
                self.peer.append(p.value)
            self.slots = []
            for p in self.ptrs:
                raw = torch.as_tensor(_DeviceBuffer(p, slot_bytes), device=self.device)
                kv = raw.view(torch.float16).view(2, self.slot_rows, heads, head_dim)
                self.slots.append(kv)
            self.copy_stream = torch.cuda.Stream(self.device)
            self.flag = torch.zeros(1, dtype=torch.int32, device=self.device)

    def share_rows(self, rank: Optional[int] = None):
        """Node rows [r0, r1) of a rank's K / V share (its slice)."""
        return self.slice_rows[self.rank if rank is None else rank]

    def run(self, Q_slab, K_share, V_share, out=None):
        import torch
        import torch.distributed as dist
        from . import api as F

        a, b = self.share_rows()
        if K_share.shape[0] != b - a or V_share.shape[0] != b - a:
            raise ValueError(f"this rank's K / V share is rows [{a}, {b})")
        cur = torch.cuda.current_stream(self.device)
        if out is None:
            out = torch.empty(Q_slab.shape, dtype=self.out_dtype, device=self.device)
        if b > a:
            self.slots[0][0, :b - a].copy_(K_share)
            self.slots[0][1, :b - a].copy_(V_share)

        held = {}

        def compute(s, j):
            # the slot is complete here (received before the last handshake):
            # the send of this step waits for this point, not for the kernel
            held[s] = torch.cuda.Event()
            held[s].record(cur)
            ja, jb = self.slice_rows[j]
            pa, pb = self.plan.piece_ranges[j]
            if pb > pa:
                kv = self.slots[s % 2]
                F.forward_pieces(Q_slab, kv[0, :max(jb - ja, 1)], kv[1, :max(jb - ja, 1)], self.fmt, self.plan,
                                 out, piece_begin=pa, piece_end=pb, kv_col_base=int(self.cuts[j]),
                                 q_window_base=self.lo, block_hints=self.hints)

        def send(s):
            j = ring_slice_at(self.rank, s, self.world)
            ja, jb = self.slice_rows[j]
            if jb <= ja:
                return
            self.copy_stream.wait_event(held[s])
            src, dst = self.ptrs[s % 2], self.peer[(s + 1) % 2]
            sp = self.copy_stream.cuda_stream
            n = (jb - ja) * self.row_bytes
            for half in range(2):  # K rows, then V rows
                off = half * self.slot_rows * self.row_bytes
                st = self.lib.f3s_peer_copy(dst + off, src + off, n, sp)
                if st != 0:
                    from . import _lib
                    raise _lib.Fused3SError(st, "f3s_peer_copy")

        def handshake(s):
            cur.wait_stream(self.copy_stream)
            dist.all_reduce(self.flag, group=self.group)

        ring_pass(self.rank, self.world, compute, send, handshake)
        F.plan_merge(self.plan, out, self.fmt.num_nodes, q_window_base=self.lo)
        return out

    def close(self):
        """Collective: unmap the next rank's slots, then free this rank's."""
        import torch
        import torch.distributed as dist

        if not self.ptrs:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self.peer:
            self.lib.f3s_peer_close(p)
        dist.barrier(group=self.group)
        self.slots = []
        for p in self.ptrs:
            self.lib.f3s_peer_free(p)
        self.ptrs, self.peer = [], []
