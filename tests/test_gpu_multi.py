"""Sharded forward with the O all-gather overlapped per sub-slab, on two GPUs
(NCCL over NVLink): the gathered O equals the 1-GPU O bit for bit.  Skipped
on a box with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    import fused3s_b200 as F
    from fused3s_b200 import graphs as G, shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        g = G.powerlaw_graph(num_nodes=6007, directed_edges=60000, max_degree=900, seed=13)
        qf, kf, vf = (t.to(dev) for t in G.make_features(g.num_nodes, 4, 64, kind="normal", seed=7))
        fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
        order = F.generate_balanced_window_order(fmt)
        off = fmt.window_offsets.cpu().numpy()
        parts = shard.partition_windows(off, world)
        r0, r1 = shard.slab_rows(*parts[rank], g.num_nodes)
        ok = []
        # pieces are cut per window (at most 8 blocks), so the planned 1-GPU
        # run and every planned slab agree bit for bit
        full_plan = F.make_plan(fmt, 4, 64, max_blocks=8)
        for dtype in (torch.float32, torch.float16):
            full = F.fused3s_forward(qf, kf, vf, fmt, out_dtype=dtype, plan=full_plan, check_status=True)
            for sub in (1, 4):
                lo, hi = parts[rank]
                subs = shard.sub_ranges(off, lo, hi, sub)
                plans = [F.make_plan(fmt, 4, 64, order=shard.rank_order(order, a, b).contiguous(), max_blocks=8)
                         for a, b in subs]
                got = shard.sharded_forward_allgather(qf[r0:r1].contiguous(), kf, vf, fmt, order, parts, rank,
                                                      window_offsets=off, sub_slabs=sub, out_dtype=dtype,
                                                      plans=plans)
                torch.cuda.synchronize()
                ok.append(bool(torch.equal(got, full)))
                # the same through the copy engines (IPC-mapped peer buffers), two steps
                pg = shard.PeerGather(off, parts, rank, g.num_nodes, (4, 64), dtype, dev, sub)
                for _ in range(2):
                    got = shard.sharded_forward_allgather(qf[r0:r1].contiguous(), kf, vf, fmt, order, parts, rank,
                                                          window_offsets=off, sub_slabs=sub, out_dtype=dtype,
                                                          plans=plans, gather=pg)
                    torch.cuda.synchronize()
                    ok.append(bool(torch.equal(got, full)))
                pg.close()
        q.put((rank, all(ok)))
    finally:
        dist.destroy_process_group()


def test_sharded_forward_allgather_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    assert sorted(results) == [(0, True), (1, True)]


def _ring_worker(rank, world, port, q):
    """K / V sharded over the ranks and passed around the ring (shard.RingKV),
    and the host-memory forward with each rank uploading only its K / V
    share (hostio.HostForward, NCCL all-gather to the replica)."""
    import datetime
    import torch.distributed as dist
    import fused3s_b200 as F
    import oracle
    from fused3s_b200 import graphs as G, shard, hostio

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        H, d = 4, 64
        g = G.powerlaw_graph(num_nodes=9001, directed_edges=90000, max_degree=1200, seed=21)
        qf, kf, vf = (t.to(dev) for t in G.make_features(g.num_nodes, H, d, kind="normal", seed=5))
        fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
        order = F.generate_balanced_window_order(fmt)
        off, cols = fmt.to_host()
        parts = shard.partition_windows(off, world)
        lo, hi = parts[rank]
        r0, r1 = shard.slab_rows(lo, hi, g.num_nodes)
        ok = []
        ring = shard.RingKV(fmt, H, d, (lo, hi), rank, world, order=order)
        a, b = ring.share_rows()
        # the same sliced plan on one GPU with the whole K / V: bit-identical
        ref_plan = F.make_sliced_plan(fmt, H, d, ring.cuts, order=shard.rank_order(order, lo, hi).contiguous())
        want = torch.empty((r1 - r0, H, d), dtype=torch.float32, device=dev)
        F.forward_pieces(qf[r0:r1].contiguous(), kf, vf, fmt, ref_plan, want, q_window_base=lo, check_status=True)
        F.plan_merge(ref_plan, want, g.num_nodes, q_window_base=lo)
        for _ in range(2):  # two steps: the slots are reused
            got = ring.run(qf[r0:r1].contiguous(), kf[a:b].contiguous(), vf[a:b].contiguous())
            torch.cuda.synchronize()
            ok.append(bool(torch.equal(got, want)))
        ring.close()
        # against the replicated-K / V forward and the oracle, within the bar
        full_o = F.fused3s_forward(qf, kf, vf, fmt, check_status=True)
        full = full_o[r0:r1]
        o = got.cpu().numpy()
        ok.append(oracle.rel_l2(o, full.cpu().numpy()) <= 1e-3)
        wins = np.arange(lo, hi, max(1, (hi - lo) // 40))
        _, ref = oracle.sampled_check(g.num_nodes, off, cols, wins, qf, kf, vf, full_o, threads=8)
        rows = np.concatenate([np.arange(16 * w, min(16 * w + 16, g.num_nodes)) for w in wins]) - r0
        ok.append(oracle.max_abs(o[rows], ref) <= 2e-2 and oracle.rel_l2(o[rows], ref) <= 1e-3)
        # host-memory forward, K / V uploaded as shares and all-gathered
        hf = hostio.HostForward(fmt, H, d, order=order, window_range=(lo, hi), kv_share=(rank, world), sub_slabs=3)
        sa, sb = hf.share_ranges[rank]
        hQ = hostio.pinned_empty((r1 - r0, H, d), torch.float16)
        hQ.copy_(qf[r0:r1])
        hK = hostio.pinned_empty((sb - sa, H, d), torch.float16)
        hK.copy_(kf[sa:sb])
        hV = hostio.pinned_empty((sb - sa, H, d), torch.float16)
        hV.copy_(vf[sa:sb])
        hO = hostio.pinned_empty((r1 - r0, H, d), torch.float32)
        for _ in range(2):
            hf.run(hQ, hK, hV, hO)
            torch.cuda.synchronize()
            ok.append(oracle.rel_l2(hO.numpy(), full.cpu().numpy()) <= 1e-3)
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_ring_kv_and_sharded_host_forward_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ring_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert all(all(v) for v in results.values()), results
