"""Host logic of the multi-GPU paths, run as gloo ranks on CPU (no GPU):

  * the ring schedule of K / V slices (shard.ring_pass) with a real message
    transport: every rank sees every slice exactly once, in the scheduled
    order, with the double-buffered slots never overwritten while in use;
  * failure detection: a rank that leaves between steps is reported to the
    survivors by the heartbeat (RankFailure) within the deadline, and a
    collective it never joins ends with CollectiveTimeout within the
    deadline instead of hanging.  The failure is made on the host (a rank
    that exits); no GPU is involved.
"""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fused3s_b200 import shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_ring_slice_schedule_covers_every_slice_once():
    for world in (1, 2, 3, 5, 8):
        for rank in range(world):
            seen = [shard.ring_slice_at(rank, s, world) for s in range(world)]
            assert sorted(seen) == list(range(world)) and seen[0] == rank
        # at every step the ranks hold distinct slices, and rank r receives
        # what rank r - 1 held
        for s in range(world - 1):
            for r in range(world):
                assert shard.ring_slice_at(r, s + 1, world) == shard.ring_slice_at((r - 1) % world, s, world)


def _ring_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rows = 37
        # slice j's payload: every element equals j (K) and 100 + j (V)
        slots = [torch.full((2, rows), -1.0) for _ in range(2)]
        slots[0][0] = rank
        slots[0][1] = 100 + rank
        seen = []
        reqs = []

        def compute(s, j):
            kv = slots[s % 2]
            ok = bool(torch.all(kv[0] == j) and torch.all(kv[1] == 100 + j))
            seen.append((s, j, ok))

        def send(s):
            nxt, prv = (rank + 1) % world, (rank - 1) % world
            reqs.append(dist.isend(slots[s % 2].clone(), nxt))
            reqs.append(dist.irecv(slots[(s + 1) % 2], prv))

        def handshake(s):
            while reqs:
                reqs.pop().wait()
            dist.barrier()

        shard.ring_pass(rank, world, compute, send, handshake)
        result_q.put((rank, seen))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_ring_pass_moves_every_slice_to_every_rank(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ring_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        seen = results[r]
        assert [j for _, j, _ in seen] == [(r - s) % world for s in range(world)]
        assert all(ok for *_, ok in seen), seen


def _exit_now(result_q):
    """Leave the process at once (no process-group teardown), after the
    queue's feeder thread has written the result out."""
    result_q.close()
    result_q.join_thread()
    os._exit(0)


def _failure_worker(rank, world, port, mode, result_q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    store = dist.distributed_c10d._get_default_store()
    hb = shard.Heartbeat(store, rank, world, deadline_s=2.0)
    slabs = [(0, 5), (5, 9), (9, 16)]
    x = torch.arange(16, dtype=torch.float32).reshape(16, 1)
    r0, r1 = slabs[rank]
    # step 0: everyone takes part
    hb.step(0)
    full = shard.gather_rows(x[r0:r1].clone(), slabs, deadline_s=10.0)
    ok0 = bool(torch.equal(full, x))
    if rank == world - 1:
        # leaves between steps: nothing of its own is in flight
        result_q.put((rank, "left", ok0, 0.0))
        _exit_now(result_q)
    t0 = time.monotonic()
    try:
        if mode == "heartbeat":
            hb.step(1)
        else:
            shard.gather_rows(x[r0:r1].clone(), slabs, deadline_s=2.0)
        outcome = "no error"
    except shard.RankFailure as e:
        outcome = f"RankFailure{e.missing}"
    except shard.CollectiveTimeout:
        outcome = "CollectiveTimeout"
    result_q.put((rank, outcome, ok0, time.monotonic() - t0))
    _exit_now(result_q)  # the group is unusable now; skip its teardown


@pytest.mark.parametrize("mode", ["heartbeat", "collective"])
def test_rank_leaving_between_steps_is_reported_within_the_deadline(mode):
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failure_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, outcome, ok0, waited = q.get(timeout=120)
        results[r] = (outcome, ok0, waited)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert results[2][0] == "left"
    want = "RankFailure[2]" if mode == "heartbeat" else "CollectiveTimeout"
    for r in (0, 1):
        outcome, ok0, waited = results[r]
        assert ok0, "step 0 must succeed on every rank"
        assert outcome == want, results
        assert waited < 10.0, f"rank {r} waited {waited:.1f}s"
