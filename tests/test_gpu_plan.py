"""Work plans: heavy windows cut into pieces whose partial softmax states are
merged after the fused kernel.  Same parity bar as every forward test
(max-abs 2e-2, rel-L2 1e-3 against the reference's CPU ground truth), and
deterministic: the merge runs in piece order."""
import numpy as np
import pytest
import torch

import oracle
import fused3s_b200 as F
from conftest import MAX_ABS_TOL, REL_L2_TOL
from fused3s_b200 import _lib
from fused3s_b200 import graphs as G

pytestmark = pytest.mark.gpu


def feats(n, h, d, kind="uniform", seed=42):
    q, k, v = G.make_features(n, h, d, kind=kind, seed=seed, device="cpu")
    return q.numpy(), k.numpy(), v.numpy()


def gpu(*a):
    return [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in a]


def parity(o, ref, what):
    ma, rl = oracle.max_abs(o, ref), oracle.rel_l2(o, ref)
    assert ma <= MAX_ABS_TOL and rl <= REL_L2_TOL, f"{what}: maxabs={ma:.3e} relL2={rl:.3e}"


@pytest.mark.parametrize("heads,head_dim,T", [(1, 64, 3), (2, 64, 5), (8, 64, 4), (4, 128, 7), (3, 64, 16)])
def test_plan_matches_oracle(lib, heads, head_dim, T):
    g = G.powerlaw_graph(num_nodes=2003, directed_edges=20000, max_degree=500, seed=heads + T)
    q, k, v = feats(g.num_nodes, heads, head_dim)
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    plan = F.make_plan(fmt, heads, head_dim, max_blocks=T)
    Q, K, V = gpu(q, k, v)
    o = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True).cpu().numpy()
    off, cols = fmt.to_host()
    assert np.diff(off).max() > T  # something was split
    ref = oracle.block_attention(g.num_nodes, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                                 off, cols, threads=8)
    parity(o, ref, f"H={heads} d={head_dim} T={T}")
    o2 = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True).cpu().numpy()
    assert np.array_equal(o, o2)  # deterministic


def test_plan_without_splits_is_bit_identical(lib):
    g = G.make_graph("c1")
    q, k, v = feats(g.num_nodes, 1, 64)
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    Q, K, V = gpu(q, k, v)
    plan = F.make_plan(fmt, 1, 64, max_blocks=1 << 20)
    a = F.fused3s_forward(Q, K, V, fmt, check_status=True).cpu()
    b = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True).cpu()
    assert torch.equal(a, b)


def test_plan_slabs_equal_full_planned(lib):
    """Per-rank plans over contiguous window slabs reproduce the full planned
    output bit for bit (the piece cut depends only on the window)."""
    g = G.powerlaw_graph(num_nodes=4099, directed_edges=40000, max_degree=800, seed=9)
    q, k, v = feats(g.num_nodes, 2, 64)
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    Q, K, V = gpu(q, k, v)
    T = 6
    full = F.fused3s_forward(Q, K, V, fmt, plan=F.make_plan(fmt, 2, 64, max_blocks=T), check_status=True).cpu()
    order = F.generate_balanced_window_order(fmt)
    parts = []
    cuts = [0, 50, 120, fmt.num_row_windows]
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        r0, r1 = 16 * lo, min(16 * hi, g.num_nodes)
        mine = order[(order >= lo) & (order < hi)].contiguous()
        plan = F.make_plan(fmt, 2, 64, order=mine, max_blocks=T)
        parts.append(F.fused3s_forward(Q[r0:r1].contiguous(), K, V, fmt, q_window_base=lo, plan=plan,
                                       check_status=True).cpu())
    assert torch.equal(torch.cat(parts), full)


def test_plan_overflow_is_reported(lib):
    """A plan sized with a too-small block bound records an error instead of
    writing past its end, and the forward refuses it."""
    g = G.make_graph("c1")
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    order = F.generate_balanced_window_order(fmt)
    n = fmt.num_row_windows
    size = lib.f3s_plan_size(n, 1, 1, 1, 64)  # claims one block in total
    buf = torch.zeros(size, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.f3s_make_plan(fmt.window_offsets.data_ptr(), order.data_ptr(), n, 1, 1, 1, 64, buf.data_ptr(), size,
                             stream) == 0
    plan = F.ForwardPlan(buf, 1, 64, 1)
    q, k, v = (t.cuda() for t in G.make_features(g.num_nodes, 1, 64))
    with pytest.raises(_lib.Fused3SError) as e:
        F.fused3s_forward(q, k, v, fmt, plan=plan, check_status=True)
    assert e.value.status == _lib.F3S_ERR_BAD_FORMAT
    F.fused3s_forward(q, k, v, fmt, check_status=True)  # device still fine


def test_plan_usable_after_failed_forward(lib):
    """A planned forward that aborts (here: plan windows outside the Q slab)
    is reported, and the same plan then gives the exact result."""
    g = G.powerlaw_graph(num_nodes=2003, directed_edges=20000, max_degree=500, seed=21)
    q, k, v = feats(g.num_nodes, 2, 64)
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    Q, K, V = gpu(q, k, v)
    plan = F.make_plan(fmt, 2, 64, max_blocks=4)
    with pytest.raises(_lib.Fused3SError) as e:
        F.fused3s_forward(Q[:160].contiguous(), K, V, fmt, plan=plan, check_status=True)
    assert e.value.status == _lib.F3S_ERR_BAD_FORMAT
    o = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True).cpu().numpy()
    off, cols = fmt.to_host()
    ref = oracle.block_attention(g.num_nodes, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                                 off, cols, threads=8)
    parity(o, ref, "plan after a failed forward")


def test_plan_many_pieces_per_window(lib):
    """Windows cut into hundreds of pieces (T = 1): the last-arriving piece
    merges them all, for both head dims."""
    for heads, head_dim in ((1, 64), (4, 128)):
        g = G.powerlaw_graph(num_nodes=3001, directed_edges=40000, max_degree=1500, seed=5 + heads)
        q, k, v = feats(g.num_nodes, heads, head_dim)
        fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
        off, cols = fmt.to_host()
        assert np.diff(off).max() > 100
        Q, K, V = gpu(q, k, v)
        plan = F.make_plan(fmt, heads, head_dim, max_blocks=1)
        o = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True).cpu().numpy()
        ref = oracle.block_attention(g.num_nodes, q.astype(np.float32), k.astype(np.float32),
                                     v.astype(np.float32), off, cols, threads=8)
        parity(o, ref, f"T=1 H={heads} d={head_dim}")
        o2 = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True).cpu().numpy()
        assert np.array_equal(o, o2)


def test_plan_windows_outside_the_slab_write_nothing_outside_o(lib):
    """A plan over all windows used with a slab that starts at window 50: the
    forward reports F3S_ERR_BAD_FORMAT and neither the fused kernel nor the
    merge writes any row outside O (guard rows around O stay untouched)."""
    g = G.powerlaw_graph(num_nodes=2003, directed_edges=20000, max_degree=500, seed=21)
    q, k, v = feats(g.num_nodes, 2, 64)
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    Q, K, V = gpu(q, k, v)
    plan = F.make_plan(fmt, 2, 64, max_blocks=4)
    lo, hi, pad = 50, 100, 64
    r0, r1 = 16 * lo, 16 * hi
    big = torch.full((r1 - r0 + 2 * pad, 2, 64), 7.0, dtype=torch.float32, device="cuda")
    out = big[pad:pad + r1 - r0]
    with pytest.raises(_lib.Fused3SError) as e:
        F.fused3s_forward(Q[r0:r1].contiguous(), K, V, fmt, plan=plan, out=out, q_window_base=lo,
                          check_status=True)
    assert e.value.status == _lib.F3S_ERR_BAD_FORMAT
    torch.cuda.synchronize()
    assert torch.all(big[:pad] == 7.0) and torch.all(big[pad + r1 - r0:] == 7.0)


@pytest.mark.parametrize("heads,head_dim,cw,T", [(2, 64, 8, 0), (8, 64, 4, 5), (4, 128, 16, 0), (1, 64, 2, 3)])
def test_column_chunked_plan_matches_oracle(lib, heads, head_dim, cw, T):
    """Host-built column-chunked plans (f3s_load_plan): same parity bar,
    deterministic, and equal to themselves on a window subset's slab."""
    g = G.powerlaw_graph(num_nodes=2003, directed_edges=20000, max_degree=500, seed=heads + cw)
    q, k, v = feats(g.num_nodes, heads, head_dim)
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    plan = F.make_chunked_plan(fmt, heads, head_dim, chunk_cols=cw, max_blocks=T)
    Q, K, V = gpu(q, k, v)
    o = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True).cpu().numpy()
    off, cols = fmt.to_host()
    ref = oracle.block_attention(g.num_nodes, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                                 off, cols, threads=8)
    parity(o, ref, f"chunked H={heads} d={head_dim} cw={cw} T={T}")
    o2 = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True).cpu().numpy()
    assert np.array_equal(o, o2)
    # a slab of windows [30, 90) with its own chunked plan: the same rows bit for bit
    lo, hi = 30, 90
    order = F.generate_balanced_window_order(fmt)
    mine = order[(order >= lo) & (order < hi)].contiguous()
    sp = F.make_chunked_plan(fmt, heads, head_dim, order=mine, chunk_cols=cw, max_blocks=T)
    r0, r1 = 16 * lo, 16 * hi
    os_ = F.fused3s_forward(Q[r0:r1].contiguous(), K, V, fmt, plan=sp, q_window_base=lo, check_status=True)
    assert np.array_equal(os_.cpu().numpy(), o[r0:r1])


def test_load_plan_rejects_out_of_range_pieces(lib):
    g = G.make_graph("c1")
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    off, cols = fmt.to_host()
    pieces, splits, n_slots, _ = F.column_chunk_pieces(off, cols, np.arange(fmt.num_row_windows), 8, 0)
    size = lib.f3s_plan_size_for(pieces.shape[0], splits.shape[0], n_slots, 1, 64)
    buf = torch.empty(size, dtype=torch.uint8, device="cuda")
    off32 = np.ascontiguousarray(off.astype(np.int32))
    stream = torch.cuda.current_stream().cuda_stream
    for bad in ((0, 2, 10**6), (0, 3, n_slots), (0, 0, fmt.num_row_windows)):
        p = pieces.copy()
        p[bad[0], bad[1]] = bad[2]
        p = np.ascontiguousarray(p)
        st = lib.f3s_load_plan(p.ctypes.data, p.shape[0], np.ascontiguousarray(splits).ctypes.data, splits.shape[0],
                               n_slots, off32.ctypes.data, fmt.num_row_windows, 1, 64, buf.data_ptr(), size, stream)
        assert st == _lib.F3S_ERR_BAD_FORMAT
