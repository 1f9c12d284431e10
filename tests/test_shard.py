"""Multi-GPU host logic on CPU: the window partition, the per-rank order and
the slab all-gather, the latter with two gloo ranks."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from fused3s_b200 import graphs as G
from fused3s_b200 import shard


def test_partition_covers_all_windows_contiguously():
    rng = np.random.default_rng(0)
    for world in (1, 2, 3, 4, 8):
        cnt = rng.zipf(1.7, 5000).clip(max=20000)
        off = np.concatenate([[0], np.cumsum(cnt)])
        parts = shard.partition_windows(off, world)
        assert len(parts) == world
        assert parts[0][0] == 0 and parts[-1][1] == 5000
        for (a, b), (c, d) in zip(parts[:-1], parts[1:]):
            assert b == c and a <= b
        cost = cnt + shard.WINDOW_COST
        loads = [cost[a:b].sum() for a, b in parts]
        # contiguous cuts are within one window's cost of the ideal share
        assert max(loads) - cost.sum() / world <= cost.max() + 1e-9


def test_partition_more_ranks_than_windows():
    off = np.array([0, 3, 5])
    parts = shard.partition_windows(off, 4)
    assert parts[0][0] == 0 and parts[-1][1] == 2
    assert sum(b - a for a, b in parts) == 2


def test_rank_orders_partition_the_global_order():
    g = G.make_graph("c2")
    off, _ = oracle.convert(g.num_nodes, g.row_ptr, g.col_ind)
    order = oracle.window_order(off)
    parts = shard.partition_windows(off, 3)
    got = [shard.rank_order(order, a, b) for a, b in parts]
    assert sorted(np.concatenate(got).tolist()) == list(range(len(off) - 1))
    cnt = np.diff(off)
    for o in got:
        assert np.all(np.diff(cnt[o]) <= 0)  # still descending


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gather_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = 1003
        full = torch.arange(n * 6, dtype=torch.float32).reshape(n, 2, 3)
        off = np.concatenate([[0], np.cumsum(np.random.default_rng(1).integers(0, 9, (n + 15) // 16))])
        parts = shard.partition_windows(off, world)
        slabs = [shard.slab_rows(a, b, n) for a, b in parts]
        r0, r1 = slabs[rank]
        got = shard.gather_rows(full[r0:r1].clone(), slabs)
        result_q.put((rank, bool(torch.equal(got, full))))
    finally:
        dist.destroy_process_group()


def test_gather_rows_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(results) == [(0, True), (1, True)]


def test_sub_ranges_cover_the_slab():
    rng = np.random.default_rng(4)
    cnt = rng.zipf(1.8, 777).clip(max=5000)
    off = np.concatenate([[0], np.cumsum(cnt)])
    for lo, hi in ((0, 777), (100, 101), (300, 300), (5, 640)):
        for parts in (1, 3, 4, 8):
            subs = shard.sub_ranges(off, lo, hi, parts)
            assert len(subs) == parts
            assert subs[0][0] == lo and subs[-1][1] == hi
            for (a, b), (c, d) in zip(subs[:-1], subs[1:]):
                assert b == c and a <= b


def _overlap_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = 1501
        rng = np.random.default_rng(2)
        off = np.concatenate([[0], np.cumsum(rng.integers(0, 30, (n + 15) // 16))])
        parts = shard.partition_windows(off, world)
        full = torch.arange(n * 6, dtype=torch.float32).reshape(n, 2, 3)
        ok = True
        for sub_slabs in (1, 3, 4):
            og = shard.OverlappedGather(off, parts, rank, n, (2, 3), torch.float32, "cpu", sub_slabs)
            r0, r1 = shard.slab_rows(*parts[rank], n)
            o_slab = torch.full((r1 - r0, 2, 3), -1.0)
            for j, (a, b) in enumerate(og.my_sub_ranges()):
                ra, rb = shard.slab_rows(a, b, n)
                o_slab[ra - r0:rb - r0] = full[ra:rb]  # the "computation" of sub-slab j
                og.send(j, o_slab)
            ok = ok and bool(torch.equal(og.finish(), full))
        result_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_overlapped_gather_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_overlap_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(results) == [(0, True), (1, True)]


def test_device_er_generator_family():
    """The vectorised C3 generator (batched_er_graph_device), run with torch
    on the CPU: block-diagonal, symmetric, every self-loop, mean degree near
    8 + 1, sizes in range, deterministic for a seed."""
    from fused3s_b200 import graphs as G
    g = G.batched_er_graph_device(num_graphs=200, device="cpu", seed=11)
    g2 = G.batched_er_graph_device(num_graphs=200, device="cpu", seed=11)
    assert np.array_equal(g.row_ptr, g2.row_ptr) and np.array_equal(g.col_ind, g2.col_ind)
    rp, ci = g.row_ptr.astype(np.int64), g.col_ind.astype(np.int64)
    deg = np.diff(rp)
    assert 8.0 < deg.mean() < 10.0
    rows = np.repeat(np.arange(g.num_nodes), deg)
    edges = set(zip(rows.tolist(), ci.tolist()))
    assert all((b, a) in edges for a, b in edges)
    assert all((i, i) in edges for i in range(g.num_nodes))
    # block diagonal: no edge crosses a component; components are 20..500 nodes
    import scipy.sparse as sp
    from scipy.sparse.csgraph import connected_components
    A = sp.csr_matrix((np.ones(ci.shape[0]), ci, rp), shape=(g.num_nodes, g.num_nodes))
    _, lab = connected_components(A, directed=False)
    sizes = np.bincount(lab)
    assert sizes.max() <= 500  # components stay inside one graph of at most 500 nodes
    assert np.all(np.abs(rows - ci) < 500)  # graphs are laid out one after another


def test_kv_share_rows_cover_k_and_v():
    """Each rank's share of K / V rows for the host-memory forward
    (hostio.kv_share_rows): whole block columns, equal padded sizes (what
    the all-gather into the replica needs), in rank order, together exactly
    the N rows, empty shares for surplus ranks."""
    from fused3s_b200 import hostio

    for n in (1, 15, 16, 17, 1000, 2708, 1 << 20):
        for world in (1, 2, 3, 4, 8):
            share, rows = hostio.kv_share_rows(n, world)
            assert share % 16 == 0 and world * share >= n
            assert len(rows) == world
            assert rows[0][0] == 0 and rows[-1][1] == n
            for (a, b), (c, d) in zip(rows[:-1], rows[1:]):
                assert b == c
            for r, (a, b) in enumerate(rows):
                assert a == min(r * share, n) and b - a <= share
                assert a % 16 == 0 or a == n
    share, rows = hostio.kv_share_rows(17, 8)  # two block columns over eight ranks
    assert share == 16 and rows[:2] == [(0, 16), (16, 17)] and all(a == b for a, b in rows[2:])
