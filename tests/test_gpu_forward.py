"""Fused forward on the GPU against the reference's CPU ground truth.

Tolerance (from the north-star specification, fp16 inputs and fp32
accumulation): max-abs error <= 2e-2 and relative L2 error <= 1e-3 against
the reference's block-semantics attention on identical (fp16-valued) inputs.
"""
import numpy as np
import pytest
import torch

import oracle
import fused3s_b200 as F
from conftest import MAX_ABS_TOL, REL_L2_TOL
from fused3s_b200 import graphs as G

pytestmark = pytest.mark.gpu


def features_np(n, h, d, kind="uniform", seed=42):
    q, k, v = G.make_features(n, h, d, kind=kind, seed=seed, device="cpu")
    return q.numpy(), k.numpy(), v.numpy()


def to_gpu(*arrs):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


def assert_parity(o, ref, what=""):
    ma, rl = oracle.max_abs(o, ref), oracle.rel_l2(o, ref)
    assert ma <= MAX_ABS_TOL and rl <= REL_L2_TOL, f"{what}: maxabs={ma:.3e} relL2={rl:.3e}"
    return ma, rl


def forward_np(n, rp, ci, q, k, v, **kw):
    fmt = F.convert_csr_to_block_sparse(n, rp, ci)
    Q, K, V = to_gpu(q, k, v)
    O = F.fused3s_forward(Q, K, V, fmt, check_status=True, **kw)
    torch.cuda.synchronize()
    return fmt, O.cpu().numpy()


def test_forward_golden_fixtures(lib, golden_attention):
    """Fixtures produced by the reference's cpu_block_sparse_attention."""
    for name, c in golden_attention.items():
        n = int(c["N"][0])
        _, o = forward_np(n, c["row_ptr"], c["col_ind"], c["Q"], c["K"], c["V"])
        assert_parity(o, c["O"], name)


@pytest.mark.parametrize("config", ["c1", "c2"])
def test_forward_small_configs_full(lib, config):
    g = G.make_graph(config)
    cfg = G.CONFIGS[config]
    q, k, v = features_np(g.num_nodes, cfg.heads, cfg.head_dim, cfg.features)
    fmt, o = forward_np(g.num_nodes, g.row_ptr, g.col_ind, q, k, v)
    off, cols = fmt.to_host()
    ref = oracle.block_attention(g.num_nodes, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                                 off, cols, threads=4)
    assert_parity(o, ref, config)


def _sample_windows(off, n_heavy, n_random, seed=0):
    cnt = np.diff(off)
    heavy = np.argsort(-cnt, kind="stable")[:n_heavy]
    rng = np.random.default_rng(seed)
    rand = rng.choice(len(cnt), size=min(n_random, len(cnt)), replace=False)
    return np.unique(np.r_[heavy, rand]).astype(np.int32)


def _check_sampled(g, q, k, v, o, fmt, n_heavy, n_random, threads=16):
    off, cols = fmt.to_host()
    wins = _sample_windows(off, n_heavy, n_random)
    ref = oracle.block_attention(g.num_nodes, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                                 off, cols, windows=wins, threads=threads)
    rows = (wins[:, None] * 16 + np.arange(16)[None, :]).reshape(-1)
    rows = rows[rows < g.num_nodes]
    return assert_parity(o[rows], ref[rows], g.name)


def test_forward_c3_sampled(lib):
    g = G.make_graph("c3")
    cfg = G.CONFIGS["c3"]
    q, k, v = features_np(g.num_nodes, cfg.heads, cfg.head_dim, cfg.features)
    fmt, o = forward_np(g.num_nodes, g.row_ptr, g.col_ind, q, k, v)
    _check_sampled(g, q, k, v, o, fmt, 32, 512)


def test_forward_c4_sampled(lib):
    g = G.make_graph("c4", device="cuda")
    cfg = G.CONFIGS["c4"]
    q, k, v = features_np(g.num_nodes, cfg.heads, cfg.head_dim, cfg.features)
    fmt, o = forward_np(g.num_nodes, g.row_ptr, g.col_ind, q, k, v)
    _check_sampled(g, q, k, v, o, fmt, 3, 128)


def test_forward_c5_family_scaled_sampled(lib):
    """C5's R-MAT family and head shape (H=4, d=128) at 2^18 nodes."""
    g = G.rmat_graph(18, 32, device="cuda", name="c5-scaled")
    q, k, v = features_np(g.num_nodes, 4, 128, "normal")
    fmt, o = forward_np(g.num_nodes, g.row_ptr, g.col_ind, q, k, v)
    _check_sampled(g, q, k, v, o, fmt, 3, 128)


@pytest.mark.parametrize("heads,head_dim", [(1, 64), (2, 64), (3, 64), (4, 64), (8, 64), (16, 64),
                                            (1, 128), (2, 128), (4, 128), (6, 128)])
def test_forward_heads_and_dims(lib, heads, head_dim):
    g = G.powerlaw_graph(num_nodes=1203, directed_edges=8000, max_degree=300, seed=heads * 7 + head_dim)
    q, k, v = features_np(g.num_nodes, heads, head_dim, "uniform", seed=heads)
    fmt, o = forward_np(g.num_nodes, g.row_ptr, g.col_ind, q, k, v)
    off, cols = fmt.to_host()
    ref = oracle.block_attention(g.num_nodes, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                                 off, cols, threads=8)
    assert_parity(o, ref, f"H={heads} d={head_dim}")


def test_forward_tail_masking(lib):
    """N % 16 != 0: columns >= N of the last block column are masked like the
    reference's CPU ground truth (the reference v2 kernel does not mask)."""
    n = 16 * 20 + 5
    rng = np.random.default_rng(1)
    s = rng.integers(0, n, 2000)
    d = rng.integers(0, n, 2000)
    d[:300] = n - 1  # many edges into the last, partial block column
    gr = G.csr_from_edges(n, s, d)
    q, k, v = features_np(n, 2, 64)
    fmt, o = forward_np(n, gr.row_ptr, gr.col_ind, q, k, v)
    off, cols = fmt.to_host()
    ref = oracle.block_attention(n, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), off, cols)
    assert_parity(o, ref, "tail")


def test_legacy_launch_matches_v2_semantics(lib):
    """f3s_1tb1rw_kernel: reference argument list, padded nrw*16 buffers, every
    padded row treated as a node (what the v2 kernel computes)."""
    g = G.make_graph("c1")
    n = g.num_nodes
    nrw = (n + 15) // 16
    rows = nrw * 16
    q, k, v = features_np(n, 1, 64)
    pad = lambda a: np.concatenate([a[:, 0, :], np.zeros((rows - n, 64), np.float16)])
    qp, kp, vp = pad(q), pad(k), pad(v)
    fmt = F.convert_csr_to_block_sparse(n, g.row_ptr, g.col_ind)
    order = F.generate_balanced_window_order(fmt)
    Q, K, V = to_gpu(qp, kp, vp)
    O = torch.zeros(rows, 64, dtype=torch.float32, device="cuda")
    F.f3s_1tb1rw_kernel(Q, K, V, O, fmt.window_offsets, fmt.block_col_indices, order, nrw, 64)
    torch.cuda.synchronize()
    off, cols = fmt.to_host()
    ref = oracle.block_attention(rows, qp.astype(np.float32), kp.astype(np.float32), vp.astype(np.float32),
                                 off, cols)[:, 0, :]
    assert_parity(O.cpu().numpy(), ref, "legacy")


def test_forward_deterministic(lib):
    g = G.make_graph("c2")
    q, k, v = features_np(g.num_nodes, 1, 64)
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    Q, K, V = to_gpu(q, k, v)
    a = F.fused3s_forward(Q, K, V, fmt).cpu()
    for _ in range(5):
        b = F.fused3s_forward(Q, K, V, fmt).cpu()
        assert torch.equal(a, b)


def test_forward_slabs_equal_full(lib):
    """Row-window slabs (the multi-GPU partition) reproduce the full output bit for bit."""
    g = G.powerlaw_graph(num_nodes=5003, directed_edges=40000, max_degree=400, seed=3)
    q, k, v = features_np(g.num_nodes, 4, 64)
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    Q, K, V = to_gpu(q, k, v)
    full = F.fused3s_forward(Q, K, V, fmt).cpu()
    nrw = fmt.num_row_windows
    cuts = [0, 37, 150, nrw]
    parts = []
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        r0, r1 = lo * 16, min(hi * 16, g.num_nodes)
        order = torch.arange(lo, hi, dtype=torch.int32, device="cuda")
        parts.append(F.fused3s_forward(Q[r0:r1].contiguous(), K, V, fmt, order=order, q_window_base=lo,
                                       check_status=True).cpu())
    assert torch.equal(torch.cat(parts), full)


def test_forward_window_subset_writes_only_its_rows(lib):
    g = G.make_graph("c1")
    q, k, v = features_np(g.num_nodes, 1, 64)
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    Q, K, V = to_gpu(q, k, v)
    full = F.fused3s_forward(Q, K, V, fmt)
    out = torch.full_like(full, 7.0)
    wins = torch.tensor([3, 0, 99], dtype=torch.int32, device="cuda")
    F.fused3s_forward(Q, K, V, fmt, order=wins, out=out, check_status=True)
    mask = torch.zeros(g.num_nodes, dtype=torch.bool)
    for w in (0, 3, 99):
        mask[w * 16:(w + 1) * 16] = True
    out, full = out.cpu(), full.cpu()
    assert torch.equal(out[mask], full[mask])
    assert bool((out[~mask] == 7.0).all())


def test_forward_graph_without_edges(lib):
    n = 77
    rp = np.zeros(n + 1, np.int32)
    q, k, v = features_np(n, 2, 64)
    _, o = forward_np(n, rp, np.zeros(0, np.int32), q, k, v)
    assert not o.any()


def test_float2half_matches_torch(lib):
    x = torch.randn(1 << 20, device="cuda") * 100
    assert torch.equal(F.float2half(x), x.half())


def test_block_hints_only_change_speed(lib):
    """L2 hints are one per block and valid (0/1/2): a block's hint is its
    column's, single-use columns are streamed, kept columns are the most
    popular; the output is bit-identical with and without hints."""
    g = G.rmat_graph(14, 16, device="cuda", name="rmat14")
    q, k, v = features_np(g.num_nodes, 8, 64, "normal")
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    Q, K, V = to_gpu(q, k, v)
    hints = F.block_hints(fmt, 8, 64, l2_fraction=0.001)
    h = hints.cpu().numpy()
    off, cols = fmt.to_host()
    assert h.shape == cols.shape
    assert set(np.unique(h)) <= {0, 1, 2}
    pop = np.bincount(cols, minlength=fmt.num_row_windows)
    # one hint per column: every block of a column carries the same value
    col_hint = np.full(fmt.num_row_windows, 255, np.int64)
    col_hint[cols] = h
    assert np.array_equal(col_hint[cols], h)
    assert np.all(h[pop[cols] == 1] == 2)
    if (h == 1).any():
        assert pop[cols][h == 1].min() >= pop[cols][h == 0].max(initial=0)
        assert pop[cols][h == 1].min() >= 2
    a = F.fused3s_forward(Q, K, V, fmt, check_status=True).cpu()
    b = F.fused3s_forward(Q, K, V, fmt, block_hints=hints, check_status=True).cpu()
    assert torch.equal(a, b)
    # a subset of windows: blocks of listed windows count only listed windows
    order = torch.arange(0, fmt.num_row_windows, 3, dtype=torch.int32, device="cuda")
    hs = F.block_hints(fmt, 8, 64, order=order, l2_fraction=0.001).cpu().numpy()
    listed = np.zeros(fmt.num_row_windows, bool)
    listed[order.cpu().numpy()] = True
    in_listed = np.repeat(listed, np.diff(off))
    pop_s = np.bincount(cols[in_listed], minlength=fmt.num_row_windows)
    assert np.all(hs[in_listed & (pop_s[cols] == 1)] == 2)


@pytest.mark.parametrize("heads,head_dim", [(1, 64), (2, 128), (4, 128)])
def test_forward_heavy_windows_split_heads(lib, heads, head_dim):
    """Consumer warps that split a window's blocks (heads < 8) on windows of
    tens of thousands of blocks: every split must see its own blocks in
    order.  A few hub rows connect to every node."""
    rng = np.random.default_rng(heads)
    n = 1 << 19
    hubs = np.arange(0, 48)  # windows 0-2: hubs linked to every 16th node
    s = np.r_[np.repeat(hubs, n // 16), rng.integers(0, n, 4 * n)]
    d = np.r_[np.tile(np.arange(0, n, 16), len(hubs)) + rng.integers(0, 16, len(hubs) * (n // 16)),
              rng.integers(0, n, 4 * n)]
    gr = G.csr_from_edges(n, s, d)
    q, k, v = features_np(n, heads, head_dim, "normal", seed=heads)
    fmt, o = forward_np(n, gr.row_ptr, gr.col_ind, q, k, v)
    off, cols = fmt.to_host()
    assert np.diff(off).max() >= n // 16
    wins = np.r_[np.arange(3), np.random.default_rng(0).choice(fmt.num_row_windows, 64, replace=False)]
    ref = oracle.block_attention(n, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), off, cols,
                                 windows=np.unique(wins).astype(np.int32), threads=16)
    rows = (np.unique(wins)[:, None] * 16 + np.arange(16)).reshape(-1)
    assert_parity(o[rows], ref[rows], f"heavy H={heads} d={head_dim}")
    again = F.fused3s_forward(*to_gpu(q, k, v), fmt, check_status=True).cpu().numpy()
    assert np.array_equal(again, o)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_half_and_bf16_output_is_rounded_fp32(lib, out_dtype):
    """fp16 / bf16 O is the fp32 O rounded to nearest-even, bit for bit (with
    and without a plan); fp16 O also meets the parity bar."""
    g = G.powerlaw_graph(num_nodes=2011, directed_edges=16000, max_degree=400, seed=8)
    for heads, head_dim in ((2, 64), (4, 128)):
        q, k, v = features_np(g.num_nodes, heads, head_dim)
        fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
        Q, K, V = to_gpu(q, k, v)
        for plan in (None, F.make_plan(fmt, heads, head_dim, max_blocks=5)):
            o32 = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True)
            o16 = F.fused3s_forward(Q, K, V, fmt, plan=plan, out_dtype=out_dtype, check_status=True)
            assert o16.dtype == out_dtype
            assert torch.equal(o16, o32.to(out_dtype))
        if out_dtype == torch.float16:
            off, cols = fmt.to_host()
            ref = oracle.block_attention(g.num_nodes, q.astype(np.float32), k.astype(np.float32),
                                         v.astype(np.float32), off, cols, threads=8)
            assert_parity(o16.float().cpu().numpy(), ref, f"fp16 O H={heads} d={head_dim}")
