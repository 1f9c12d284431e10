"""Benchmark of the fused 3S hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5] [--impl ours|reference]
                    [--heads H] [--dim D] [--seed S] [--graph-seed G]
    torchrun --nproc-per-node N bench.py --gpus N ...

The default workload is C5, the largest configuration (R-MAT 2^24 nodes,
~521 M edges, 4 heads, d = 128): the one the scaling target is stated on.
A step is one fused forward (SDDMM + online softmax + SpMM) over every row
window of the graph, all heads, inputs resident in HBM.  Metric: GEdges*heads/s
= E * H / t_step (E = CSR nnz).  The graph is converted and ordered once
before timing (it is static across steps, as in a GNN layer); the converter
and order times are reported beside the metric.

With N > 1 GPUs the row windows are sharded (contiguous, cost-balanced),
K / V replicated, the fixed graph split across ranks (strong scaling); the
step time is the max over ranks of device time.  `e2e` runs the public
host-memory forward (fused3s_b200.hostio.HostForward): per step, pinned host
Q / K / V -> device (at N > 1 each rank uploads only its 1/N share of K / V,
all-gathered over NVLink), forward, O -> pinned host.

At N = 1 the cpu_baseline leg times the reference's own CPU function on a
seeded window sample and checks the timed output against the oracle on a
seeded sample of windows (`parity`); a parity failure exits non-zero.

--impl reference times the reference's own CPU implementation
(cpu_block_sparse_attention, tests/test_fused_3s_v2.cu:17, compiled from its
sources into oracle/_ref) with all host threads on a bounded, seeded sample of
windows per step, extrapolated to the full step by block count.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GEdges*heads/s"
UNIT = "GEdges*heads/s"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


_RESULT_OUT = None


def emit(record: dict) -> None:
    """Write the one JSON result line to the process's real stdout."""
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    out.write(json.dumps(record) + "\n")
    out.flush()


def route_stdout_to_stderr() -> None:
    """Keep the real stdout for the result line only: file descriptor 1 is
    pointed at stderr so banners printed by libraries (NCCL's version line,
    for one) cannot mix with it."""
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = sys.stderr


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def lib_is_default() -> bool:
    """The library in use is the package's own build (not a FUSED3S_LIB override)."""
    from fused3s_b200 import _lib
    return Path(_lib.LIB_PATH).resolve() == (ROOT / "fused3s_b200" / "libfused3s.so").resolve()


def ncu_traffic(config: str, heads: int, dim: int, split: str, order: str, hints: str):
    """DRAM bytes (read + write) per fused-kernel launch of this exact
    workload, from the committed ncu summary (a one-pass capture of the
    full-size launch), or None."""
    p = ROOT / "profiles" / "k_fused3s_dram_traffic.md"
    if not p.exists():
        return None
    key = re.escape(f"dram_bytes_per_launch[{config},H{heads},d{dim},{split},{order},hints-{hints}]")
    m = re.search(key + r":\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.proc = None
        self.gpu_id = gpu_id

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", self.gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# workload
# ----------------------------------------------------------------------------

def workload(args):
    """The configuration's shape with the command line's overrides: (cfg,
    heads, head_dim)."""
    from fused3s_b200 import graphs as G
    cfg = G.CONFIGS[args.config]
    return cfg, (args.heads or cfg.heads), (args.dim or cfg.head_dim)


def build_graph(args, device):
    from fused3s_b200 import graphs as G
    t0 = time.time()
    dev = str(device) if (device is not None and args.config in ("c4", "c5", "c4s", "c5s", "c5m")) else "cpu"
    g = G.make_graph(args.config, device=dev, seed=args.graph_seed)
    log(f"[bench] graph {args.config}: N={g.num_nodes} E={g.num_edges} ({time.time() - t0:.1f}s)")
    return g


def alg_bytes(heads, d, B, nrw, o_bytes=4):
    """Algorithmic HBM bytes of one forward: per head, K and V tiles of every
    active block (64*d B), the Q tile (32*d B) and O tile (16*d*o_bytes B:
    64*d for fp32 O) of every window; plus the block-column list and window
    offsets."""
    return heads * (64 * d * B + (32 + 16 * o_bytes) * d * nrw) + 4 * B + 8 * nrw


def alg_flops(heads, d, B):
    return 1024 * d * heads * B


# ----------------------------------------------------------------------------
# CPU baseline (reference's own cpu_block_sparse_attention, or the port)
# ----------------------------------------------------------------------------

def cpu_sample_run(num_nodes, off, cols, features, budget_s, seed, threads):
    """Run the reference CPU function on a seeded random sample of windows,
    head 0, sized to ~budget_s seconds; returns (seconds, sampled blocks,
    windows, kind).  The sample runs as its compact sub-problem (only its
    windows and the K / V blocks they use, oracle.compact_windows: the same
    arithmetic), so the largest graphs need no full-size host copy;
    features(rows) returns float32 (q, k, v) [len(rows), 1, d] of head 0 with
    zeros where rows < 0."""
    import oracle
    kind = "reference" if oracle.ref_available() else "port"
    cnt = np.diff(off)
    rng = np.random.default_rng(seed)
    perm = rng.permutation(len(cnt))
    nonempty = perm[cnt[perm] > 0]

    def run(wins):
        c = oracle.compact_windows(num_nodes, off, cols, wins)
        q, _, _ = features(c["q_rows"])
        _, k, v = features(c["kv_rows"])
        q, k, v = q[:, 0, :], k[:, 0, :], v[:, 0, :]
        t = time.perf_counter()
        if kind == "reference":
            oracle.ref_block_attention(c["num_nodes"], q, k, v, c["offsets"], c["cols"], windows=c["windows"],
                                       threads=threads)
        else:
            oracle.block_attention(c["num_nodes"], q, k, v, c["offsets"], c["cols"], windows=c["windows"],
                                   threads=threads)
        return time.perf_counter() - t

    # calibrate on a small sample, then size the real one
    n0 = min(len(nonempty), max(threads * 4, 64))
    w0 = np.sort(nonempty[:n0]).astype(np.int32)
    t0 = run(w0)
    per_block = max(t0, 1e-4) / max(int(cnt[w0].sum()), 1)
    want_blocks = budget_s / per_block
    csum = np.cumsum(cnt[nonempty])
    n1 = int(min(len(nonempty), max(n0, np.searchsorted(csum, want_blocks) + 1)))
    w1 = np.sort(nonempty[:n1]).astype(np.int32)
    t1 = run(w1)
    return t1, int(cnt[w1].sum()), n1, kind


def device_features(Q, K, V, head=0):
    """features() for cpu_sample_run from device tensors [N, H, d]."""
    import oracle

    def f(rows):
        return tuple(oracle.gather_device_rows(x, rows, head) for x in (Q, K, V))
    return f


def parity_sample(num_nodes, off, cols, Q, K, V, O, seed, threads, n_random=64, n_heavy=3):
    """The timed output against the oracle on a seeded sample: n_random
    random windows x every head against the reference's float32 CPU function
    (oracle port), and the n_heavy heaviest windows x head 0 against the same
    block semantics in float64 (over the millions of columns of a hub window
    the reference's float32 softmax sum drifts); each part within the bar."""
    import oracle
    import torch
    cnt = np.diff(off)
    rng = np.random.default_rng(seed)
    rand = np.unique(rng.choice(len(cnt), min(n_random, len(cnt)), replace=False))
    heavy = np.sort(np.argsort(-cnt, kind="stable")[:n_heavy])
    g1, w1 = oracle.sampled_check(num_nodes, off, cols, rand, Q, K, V, O, threads=threads)
    g2, w2, r2 = [], [], []
    for w in heavy:
        rows = torch.arange(16 * int(w), min(16 * int(w) + 16, num_nodes), device=Q.device)
        w2.append(oracle.block_attention_exact(num_nodes, Q[rows, 0, :].float().cpu().numpy(), K[:, 0, :],
                                               V[:, 0, :], off, cols, int(w)))
        g2.append(O[rows, 0, :].float().cpu().numpy())
    g2, w2 = np.concatenate(g2), np.concatenate(w2)
    part = {"random": (oracle.max_abs(g1, w1), oracle.rel_l2(g1, w1)),
            "heaviest": (oracle.max_abs(g2, w2), oracle.rel_l2(g2, w2))}
    return {"max_abs": max(v[0] for v in part.values()), "rel_l2": max(v[1] for v in part.values()),
            "by_part": {k: {"max_abs": v[0], "rel_l2": v[1]} for k, v in part.items()},
            "windows": int(rand.shape[0] + heavy.shape[0]),
            "sample": f"{rand.shape[0]} seeded random windows x all heads against the reference's float32 CPU "
                      f"function; the {heavy.shape[0]} heaviest windows ({cnt[heavy].tolist()} blocks) x head 0 "
                      f"against the same block semantics in float64",
            "tolerance": {"max_abs": 2e-2, "rel_l2": 1e-3}}


# ----------------------------------------------------------------------------
# arms
# ----------------------------------------------------------------------------

def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    import torch
    from fused3s_b200 import graphs as G
    import oracle
    cfg, H, d = workload(args)
    has_gpu = torch.cuda.is_available()
    g = build_graph(args, "cuda" if has_gpu else None)
    threads = os.cpu_count() or 1
    # the format from the converter restatement (bit-identical to the
    # reference's converter, tests/test_oracle.py), threaded: the timed part
    # is the reference's attention function
    off, cols = oracle.convert(g.num_nodes, g.row_ptr, g.col_ind, threads=threads)
    B, nrw = int(cols.shape[0]), len(off) - 1
    if has_gpu:  # inputs drawn on the device (the values do not change the CPU time)
        Q, K, V = G.make_features_device(g.num_nodes, 1, d, cfg.features, args.seed, "cuda")
        features = device_features(Q, K, V)
    else:
        qh, kh, vh = (x.float().numpy() for x in G.make_features(g.num_nodes, 1, d, kind=cfg.features,
                                                                    seed=args.seed))

        def features(rows):
            return tuple(oracle.gather_rows(x, rows) for x in (qh, kh, vh))
    samples = []
    for step in range(args.warmup + args.steps):
        t, blocks, nw, kind = cpu_sample_run(g.num_nodes, off, cols, features, args.ref_step_budget, seed=step,
                                             threads=threads)
        full_s = t * (B * H) / max(blocks, 1)
        if step >= args.warmup:
            samples.append(full_s)
    full_s = statistics.median(samples)
    value = g.num_edges * H / full_s / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": full_s * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config, "description": cfg.description, "num_nodes": g.num_nodes,
                   "num_edges": g.num_edges, "heads": H, "head_dim": d, "blocks": B, "row_windows": nrw},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"per step: seeded random windows of head 0 sized to ~{args.ref_step_budget:.0f}s "
                                   f"of CPU work ({blocks} of {B} blocks), time extrapolated by block count "
                                   f"to all {B} blocks x {H} heads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


def time_launches(fn, n, stream):
    """Median device time (ms) of fn() over n launches, each bracketed by its
    own events; a device-side sleep before each lets the host enqueue the
    launch before the first event is reached."""
    import torch
    times = []
    for _ in range(n):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(2_000_000)
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.median(times)


def run_ours(args):
    import torch
    import torch.distributed as dist
    import fused3s_b200 as F
    from fused3s_b200 import _lib, shard, hostio
    from fused3s_b200 import graphs as G

    rank, world, local = dist_env()
    if world > 1:
        # keep stdout to the one JSON line: no NCCL version banner
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", torch.cuda.current_device())
    lib = _lib.load()
    cfg, H, d = workload(args)
    g = build_graph(args, dev)
    N, E = g.num_nodes, g.num_edges

    # format: converted and ordered once (timed separately, not part of the step)
    rp = torch.from_numpy(g.row_ptr).to(dev)
    ci = torch.from_numpy(g.col_ind).to(dev)
    F.convert_csr_to_block_sparse(N, rp, ci)  # warm the converter
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    fmt = F.convert_csr_to_block_sparse(N, rp, ci)
    convert_ms = (time.perf_counter() - t0) * 1e3
    t0 = time.perf_counter()
    order = F.generate_balanced_window_order(fmt)
    torch.cuda.synchronize()
    order_ms = (time.perf_counter() - t0) * 1e3
    del rp, ci
    B, nrw = fmt.num_blocks, fmt.num_row_windows
    off_h = fmt.window_offsets.cpu().numpy()

    parts = shard.partition_windows(off_h, world)
    lo, hi = parts[rank]
    r0, r1 = shard.slab_rows(lo, hi, N)
    my_order = shard.rank_order(order, lo, hi).contiguous()
    if args.order == "local":
        # heavy windows first, then the rest in id order (L2 reuse between
        # neighbouring windows); heavy = above the plan's piece size
        my_blocks_all = int((fmt.window_offsets[1:] - fmt.window_offsets[:-1])[lo:hi].sum().item())
        my_order = F.locality_order(fmt, F.auto_piece_blocks(my_blocks_all, dev), order=my_order)
    Qf, Kf, Vf = G.make_features_device(N, H, d, cfg.features, args.seed, dev)
    Q = Qf[r0:r1].contiguous()
    del Qf
    o_torch = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[args.out_dtype]
    o_code = {"f32": _lib.F3S_OUT_F32, "f16": _lib.F3S_OUT_F16, "bf16": _lib.F3S_OUT_BF16}[args.out_dtype]
    O = torch.empty((r1 - r0, H, d), dtype=o_torch, device=dev)
    ws = F.forward_workspace(dev)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    n_items = int(my_order.numel())
    # L2 eviction hints per block: computed once per graph and rank
    hints = None
    hints_ms = None
    if args.l2_hints == "on":
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        hints = F.block_hints(fmt, H, d, order=my_order, l2_fraction=args.l2_keep)
        torch.cuda.synchronize()
        hints_ms = (time.perf_counter() - t0) * 1e3
    hints_ptr = hints.data_ptr() if hints is not None else None
    # work plan: heavy windows cut into pieces (computed once per graph and rank)
    plan = None
    plan_ms = None
    if args.split != "off":
        my_blocks_total = int((fmt.window_offsets[1:] - fmt.window_offsets[:-1])[lo:hi].sum().item())
        chunked = args.split.startswith("chunked")
        if args.split == "auto" or chunked or args.split.startswith("sweep"):
            T = F.auto_piece_blocks(my_blocks_total, dev)
        else:
            T = int(args.split)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        if args.split.startswith("sweep"):
            # sweep plan: windows cut at block-column chunks, the chunks swept
            # in order, one running state per window ("sweep" or
            # "sweep:<block columns per chunk>")
            chunk_cols = int(args.split.split(":")[1]) if ":" in args.split else None
            plan = F.make_sweep_plan(fmt, H, d, order=my_order, chunk_cols=chunk_cols, window_range=(lo, hi))
            ws = torch.zeros(lib.f3s_sweep_workspace_size(r1 - r0, H), dtype=torch.uint8, device=dev)
        elif chunked:
            # column-chunked plan: all SMs sweep one L2-sized range of block
            # columns at a time ("chunked" or "chunked:<block columns>")
            chunk_cols = int(args.split.split(":")[1]) if ":" in args.split else None
            plan = F.make_chunked_plan(fmt, H, d, order=my_order, chunk_cols=chunk_cols, max_blocks=T)
        else:
            plan = F.make_plan(fmt, H, d, order=my_order, max_blocks=T)
        torch.cuda.synchronize()
        plan_ms = (time.perf_counter() - t0) * 1e3
    plan_ptr = plan.buffer.data_ptr() if plan is not None else None

    def step():
        # launches on the current stream (the capture stream while a graph
        # is being recorded)
        st = lib.f3s_forward_ex(Q.data_ptr(), Kf.data_ptr(), Vf.data_ptr(), O.data_ptr(), o_code,
                                fmt.window_offsets.data_ptr(), fmt.cols_ptr, my_order.data_ptr(), hints_ptr,
                                plan_ptr, n_items, N, H, d, lo, r1 - r0, ws.data_ptr(), ws.numel(),
                                torch.cuda.current_stream(dev).cuda_stream)
        if st != 0:
            raise _lib.Fused3SError(st, "f3s_forward_ex")

    for _ in range(args.warmup):
        step()
    st = lib.f3s_workspace_status(ws.data_ptr(), sptr)
    if st != 0:
        raise _lib.Fused3SError(st, "f3s_forward (device, warm-up)")
    # The step as a CUDA graph (workspace reset + fused kernel + merge), so
    # small graphs are not bound by host launch latency.
    run = step
    graph = None
    if args.graph == "on":
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            step()
        stream.wait_stream(side)
        with torch.cuda.graph(graph):
            step()
        torch.cuda.synchronize()
        run = graph.replay

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        uuid = str(dev.index)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(uuid) as clk:
        evs[0].record(stream)
        for i in range(args.steps):
            run()
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = evs[0].elapsed_time(evs[-1])
    st = lib.f3s_workspace_status(ws.data_ptr(), sptr)
    if st != 0:
        raise _lib.Fused3SError(st, "f3s_forward (device, timed)")
    if world > 1:
        t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = E * H / (ms_per_step / 1e3) / 1e9

    threads = os.cpu_count() or 1
    cpu = None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # cpu_baseline leg: the timed O against the oracle on a seeded
        # sample, then the reference's CPU function timed on a bounded sample
        off_np, cols_np = fmt.to_host()
        t0 = time.perf_counter()
        parity = parity_sample(N, off_np, cols_np, Q, Kf, Vf, O, seed=args.seed, threads=threads)
        parity["seconds"] = time.perf_counter() - t0
        parity["ok"] = bool(parity["max_abs"] <= 2e-2 and parity["rel_l2"] <= 1e-3)
        t, blocks, nw, kind = cpu_sample_run(N, off_np, cols_np, device_features(Q, Kf, Vf), args.cpu_budget, 0,
                                             threads)
        full_s = t * (B * H) / max(blocks, 1)
        cpu = {"value": E * H / full_s / 1e9, "unit": UNIT, "cores": threads, "kind": kind,
               "sample": f"{nw} seeded random windows of head 0 ({blocks} of {B} blocks, {t:.1f}s on "
                         f"{threads} threads), extrapolated by block count to {B} blocks x {H} heads"}
        del off_np, cols_np

    # the fused kernel alone (its own events, no merge) and the merge alone
    kernel_ms, merge_ms = None, None
    if plan is not None:
        def pieces():
            st = lib.f3s_forward_pieces(Q.data_ptr(), Kf.data_ptr(), Vf.data_ptr(), O.data_ptr(), o_code,
                                        fmt.window_offsets.data_ptr(), fmt.cols_ptr, hints_ptr, plan_ptr, 0, -1, 0,
                                        N, N, H, d, lo, r1 - r0, ws.data_ptr(), ws.numel(), stream.cuda_stream)
            if st != 0:
                raise _lib.Fused3SError(st, "f3s_forward_pieces")

        def merge():
            st = lib.f3s_plan_merge(plan_ptr, O.data_ptr(), o_code, N, H, d, lo, r1 - r0, stream.cuda_stream)
            if st != 0:
                raise _lib.Fused3SError(st, "f3s_plan_merge")
        kernel_ms = time_launches(pieces, max(3, min(args.steps, 10)), stream)
        merge_ms = time_launches(merge, max(3, min(args.steps, 10)), stream)
    else:
        kernel_ms = time_launches(step, max(3, min(args.steps, 10)), stream)
    st = lib.f3s_workspace_status(ws.data_ptr(), sptr)
    if st != 0:
        raise _lib.Fused3SError(st, "f3s_forward (device, kernel timing)")

    # end to end through the public host-memory API (hostio.HostForward):
    # pinned host Q slab and K / V (this rank's share at N > 1) -> device,
    # forward, O slab -> pinned host, every step
    e2e = None
    if not args.no_e2e:
        kv_share = (rank, world) if world > 1 else None
        # one GPU: the resident buffers serve as the device side (their
        # contents are re-uploaded from the host every step)
        hf_order = order
        if args.order == "local":
            hf_order = F.locality_order(fmt, F.auto_piece_blocks(B, dev))
        hf = hostio.HostForward(fmt, H, d, order=hf_order, window_range=(lo, hi), kv_share=kv_share,
                                block_hints=hints, sub_slabs=args.sub_slabs, out_dtype=o_torch,
                                buffers=(Q, Kf, Vf, O) if world == 1 else None)
        a, b = hf.share_ranges[hf.rank]
        need = hf.h2d_bytes + hf.d2h_bytes
        try:
            import psutil
            room = psutil.virtual_memory().available
        except Exception:
            room = None
        if room is not None and need > 0.6 * room:
            log(f"[bench] e2e skipped: {need / 1e9:.1f} GB of pinned host buffers, {room / 1e9:.1f} GB free")
        else:
            hQ = hostio.pinned_empty(Q.shape, torch.float16)
            hQ.copy_(Q)
            hK = hostio.pinned_empty((b - a, H, d), torch.float16)
            hK.copy_(Kf[a:b])
            hV = hostio.pinned_empty((b - a, H, d), torch.float16)
            hV.copy_(Vf[a:b])
            torch.cuda.synchronize()
            hO = hostio.pinned_empty(O.shape, o_torch)
            e2e_steps = args.steps if ms_per_step < 1000 else max(3, min(args.steps, 5))
            hf.run(hQ, hK, hV, hO)  # warm-up
            ee = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            ee[0].record(stream)
            for _ in range(e2e_steps):
                hf.run(hQ, hK, hV, hO)
            ee[1].record(stream)
            torch.cuda.synchronize()
            e2e_ms = ee[0].elapsed_time(ee[1])
            if world > 1:
                t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                e2e_ms = float(t.item())
            e2e_step_ms = e2e_ms / e2e_steps
            e2e = {"value": E * H / (e2e_step_ms / 1e3) / 1e9, "unit": UNIT, "ms_per_step": e2e_step_ms,
                   "steps": e2e_steps, "h2d_bytes_per_step": int(hf.h2d_bytes), "d2h_bytes_per_step": int(hf.d2h_bytes),
                   "note": "per rank: pinned host Q slab + " +
                           ("its 1/N share of K and V (NCCL all-gather to the replica)" if world > 1 else "K + V") +
                           f" -> device, fused forward in {args.sub_slabs} overlapped sub-slabs, O slab -> host"}
            del hQ, hK, hV, hO
        del hf

    # optional all-gather of O (only when the full output is needed on every
    # rank): (1) after the forward, one padded all-gather; (2) the forward in
    # --sub-slabs launches, each sub-slab's all-gather overlapping the next
    # launch (shard.sharded_forward_allgather)
    gather_ms = None
    overlap_ms = None
    peer_ms = None
    if world > 1 and args.gather:
        slabs = [shard.slab_rows(a, b, N) for a, b in parts]
        ge = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        shard.gather_rows(O, slabs)
        dist.barrier()
        torch.cuda.synchronize()
        ge[0].record(stream)
        full_o = shard.gather_rows(O, slabs)
        ge[1].record(stream)
        torch.cuda.synchronize()
        gather_ms = ge[0].elapsed_time(ge[1])
        del full_o
        subs = shard.sub_ranges(off_h, lo, hi, args.sub_slabs)
        sub_plans = None
        if plan is not None:
            # piece size from each sub-slab's own blocks (a quarter of an SM's share)
            sub_plans = [F.make_plan(fmt, H, d, order=shard.rank_order(order, a, b).contiguous()) for a, b in subs]
        og = shard.OverlappedGather(off_h, parts, rank, N, (H, d), O.dtype, dev, args.sub_slabs)

        def fwd_gather():
            return shard.sharded_forward_allgather(Q, Kf, Vf, fmt, order, parts, rank, window_offsets=off_h,
                                                   sub_slabs=args.sub_slabs, out_dtype=O.dtype, block_hints=hints,
                                                   plans=sub_plans, gather=og)

        # the NCCL all-gather's kernels need SMs: time it with the forward
        # leaving k SMs free (f3s_set_forward_sm_limit) for each k asked for
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        overlap_by_free = {}
        for k in [int(x) for x in args.gather_free_sms.split(",")]:
            F.set_forward_sm_limit(sms - k if k > 0 else 0, dev)
            for _ in range(2):
                fwd_gather()
            dist.barrier()
            torch.cuda.synchronize()
            ge[2].record(stream)
            for _ in range(args.steps):
                fwd_gather()
            ge[3].record(stream)
            torch.cuda.synchronize()
            t = torch.tensor([ge[2].elapsed_time(ge[3]) / args.steps], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            overlap_by_free[k] = float(t.item())
        F.set_forward_sm_limit(0, dev)
        overlap_ms = min(overlap_by_free.values())
        del og
        # (3) the same with the rows moved by the copy engines into IPC-mapped
        # peer buffers (no SMs taken from the fused kernel)
        og = shard.PeerGather(off_h, parts, rank, N, (H, d), O.dtype, dev, args.sub_slabs)
        for _ in range(2):
            fwd_gather()
        dist.barrier()
        torch.cuda.synchronize()
        ge[2].record(stream)
        for _ in range(args.steps):
            fwd_gather()
        ge[3].record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([ge[2].elapsed_time(ge[3]) / args.steps], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        peer_ms = float(t.item())
        og.close()
        del og

    # roofline of the fused kernel (per launch, this rank's share)
    my_blocks = int((off_h[1:] - off_h[:-1])[lo:hi].sum())
    my_windows = hi - lo
    bytes_launch = alg_bytes(H, d, my_blocks, my_windows, O.element_size())
    flops_launch = alg_flops(H, d, my_blocks)
    # compulsory DRAM bytes: every input and output byte once (Q slab, the
    # K / V replica, O slab, the format)
    compulsory = ((r1 - r0) * H * d * 2 + 2 * N * H * d * 2 + (r1 - r0) * H * d * O.element_size()
                  + 4 * my_blocks + 4 * (nrw + 1) + (my_blocks if hints is not None else 0))
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    # the peak of the tensor instruction the kernel issues (mma.sync), measured
    # here on this GPU: 16 warps per SM, 8 independent chains each
    mma_tflops = _lib.ctypes.c_double(0.0)
    st = lib.f3s_probe_mma_sync(16, 4096, mma_tflops, stream.cuda_stream)
    mma_peak = mma_tflops.value if st == 0 else None
    achieved = bytes_launch / (kernel_ms / 1e3) / 1e9
    traffic = ncu_traffic(args.config, H, d, args.split, args.order, args.l2_hints) if (
        world == 1 and args.graph_seed is None and args.l2_keep == 0.5 and args.seed == 42 and lib_is_default()) \
        else None

    result = None
    if rank == 0:
        clocks = clk.summary()
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "alg_frac": achieved / hbm_peak, "traffic": traffic,
                "peak_kind": peak_kind,
                "alg_bytes_per_launch": bytes_launch, "compulsory_bytes": compulsory,
                "kernel_ms": kernel_ms, "merge_ms": merge_ms,
                "note": "achieved/frac (= alg_frac): algorithmic bytes (every block's K and V tiles, Q and O "
                        "tiles) over the fused kernel's own event time, not DRAM bytes; L2 hits let it exceed the "
                        "copy bandwidth. dram_frac: ncu DRAM bytes of the same launch (one-pass capture, "
                        "profiles/k_fused3s_dram_traffic.md) over the same time; absent where not captured.",
                "tensor_tflops": flops_launch / (kernel_ms / 1e3) / 1e12, "tensor_peak": tc_peak,
                "tensor_frac": flops_launch / (kernel_ms / 1e3) / 1e12 / tc_peak,
                "mma_sync_peak_tflops": mma_peak,
                "mma_sync_frac": (flops_launch / (kernel_ms / 1e3) / 1e12 / mma_peak) if mma_peak else None}
        if traffic is not None:
            roof["dram_gbs"] = traffic / (kernel_ms / 1e3) / 1e9
            roof["dram_frac"] = roof["dram_gbs"] / hbm_peak
            roof["traffic_over_compulsory"] = traffic / compulsory
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": args.config, "description": cfg.description, "num_nodes": N, "num_edges": E,
                       "heads": H, "head_dim": d, "blocks": B, "row_windows": nrw, "feature_seed": args.seed,
                       "graph_seed": args.graph_seed,
                       "parallelism": f"row-window shards x{world}, K/V replicated",
                       "l2": "inputs larger than L2" if (Kf.numel() + Vf.numel()) * 2 > 126e6 else
                             "inputs fit in L2 (no flush)",
                       "convert_ms": convert_ms, "order_ms": order_ms, "l2_hints": args.l2_hints,
                       "cuda_graph": args.graph, "o_dtype": args.out_dtype, "l2_keep": args.l2_keep,
                       "order": args.order,
                       "precision": "f16 Q/K/V and P on the tensor cores, f32 accumulation and softmax state",
                       "hints_ms": hints_ms, "split": args.split,
                       "piece_blocks": plan.max_blocks if plan is not None else None, "plan_ms": plan_ms},
            "roofline": roof,
            "cpu_baseline": cpu,
            "parity": parity,
            "e2e": e2e,
            "gpu_launches": args.steps * (2 if plan is not None else 1),
            "clocks": clocks,
        }
        if gather_ms is not None:
            result["allgather_o_ms"] = gather_ms
            result["forward_then_allgather_ms"] = ms_per_step + gather_ms
            result["forward_allgather_overlapped_ms"] = overlap_ms
            result["forward_allgather_overlapped_ms_by_free_sms"] = overlap_by_free
            result["forward_peer_copy_overlapped_ms"] = peer_ms
            result["sub_slabs"] = args.sub_slabs
        emit(result)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if parity is not None and not parity["ok"]:
        log(f"[bench] PARITY FAILED: {parity}")
        return 3
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c5", choices=["c1", "c2", "c3", "c4", "c5", "c4s", "c5s", "c5m"])
    ap.add_argument("--heads", type=int, default=None, help="heads (default: the configuration's)")
    ap.add_argument("--dim", type=int, default=None, choices=[64, 128], help="head dim (default: the configuration's)")
    ap.add_argument("--seed", type=int, default=42, help="seed of the Q / K / V draws")
    ap.add_argument("--graph-seed", type=int, default=None, help="seed of the graph (default: the configuration's)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--gather", action="store_true", help="also time the NCCL all-gather of O (N > 1)")
    ap.add_argument("--gather-free-sms", default="0,4,8",
                    help="SMs the forward leaves free for the overlapped NCCL all-gather (comma list, --gather)")
    ap.add_argument("--sub-slabs", type=int, default=4,
                    help="sub-slabs per rank for the overlapped forward + all-gather (--gather)")
    ap.add_argument("--out-dtype", default="f32", choices=["f32", "f16", "bf16"], help="element type of O")
    ap.add_argument("--graph", default="on", choices=["on", "off"],
                    help="replay the timed step as a CUDA graph")
    ap.add_argument("--split", default="auto",
                    help="cut windows above this many blocks into pieces: auto, off, a number, "
                         "chunked[:block columns] (pieces cut at column-chunk boundaries, swept chunk by chunk, "
                         "partial states merged after), or sweep[:block columns] (the same schedule with one "
                         "running state per window)")
    ap.add_argument("--l2-hints", default="on", choices=["on", "off"],
                    help="per block L2 eviction hints (computed once per graph)")
    ap.add_argument("--order", default="balanced", choices=["balanced", "local"],
                    help="work order: descending block count (the reference's), or heavy windows first and the "
                         "rest in id order (L2 reuse between neighbouring windows)")
    ap.add_argument("--l2-keep", type=float, default=0.5,
                    help="fraction of the L2 given to the most popular block columns (evict-last hints)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU work for cpu_baseline")
    ap.add_argument("--ref-step-budget", type=float, default=3.0, help="seconds of CPU work per reference step")
    args = ap.parse_args(argv)
    route_stdout_to_stderr()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
