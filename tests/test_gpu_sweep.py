"""Sweep plans (f3s_load_sweep_plan): windows cut at block-column chunk
boundaries, the chunks swept one after another, each window's running
softmax state carried from piece to piece inside one launch.  The result must
meet the oracle's bar on every window, equal (within the bar) the plain
forward, repeat bit for bit, and handle windows without blocks, the masked
tail, head groups with split warps, d = 128, fp16 O and a slab of windows."""
import numpy as np
import pytest
import torch

import oracle
import fused3s_b200 as F
from conftest import MAX_ABS_TOL, REL_L2_TOL
from fused3s_b200 import graphs as G

pytestmark = pytest.mark.gpu


def _graph(n, seed):
    rng = np.random.default_rng(seed)
    src = rng.integers(0, n, 12 * n)
    src[src // 16 % 9 == 0] = 3  # windows without blocks
    return G.csr_from_edges(n, src, rng.integers(0, n, 12 * n))


@pytest.mark.parametrize("n,heads,d,chunk", [(4099, 8, 64, 16), (3001, 4, 128, 32), (2051, 2, 64, 7),
                                              (5003, 1, 128, 64), (4099, 8, 64, 1)])
def test_sweep_plan_matches_the_oracle(lib, n, heads, d, chunk):
    g = _graph(n, n + heads)
    q, k, v = G.make_features(n, heads, d, kind="normal", seed=n)
    Q, K, V = q.cuda(), k.cuda(), v.cuda()
    fmt = F.convert_csr_to_block_sparse(n, g.row_ptr, g.col_ind)
    plan = F.make_sweep_plan(fmt, heads, d, chunk_cols=chunk)
    O1 = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True)
    O2 = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True)
    torch.cuda.synchronize()
    assert torch.equal(O1, O2)  # deterministic: the pieces of a window fold in in column order
    off, cols = fmt.to_host()
    ref = oracle.block_attention(n, q.float().numpy(), k.float().numpy(), v.float().numpy(), off, cols, threads=8)
    o = O1.cpu().numpy()
    ma, rl = oracle.max_abs(o, ref), oracle.rel_l2(o, ref)
    assert ma <= MAX_ABS_TOL and rl <= REL_L2_TOL, f"maxabs={ma:.3e} relL2={rl:.3e}"
    plain = F.fused3s_forward(Q, K, V, fmt, check_status=True).cpu().numpy()
    assert oracle.rel_l2(o, plain) <= REL_L2_TOL
    O16 = F.fused3s_forward(Q, K, V, fmt, plan=plan, out_dtype=torch.float16, check_status=True)
    assert torch.equal(O16, O1.to(torch.float16))


def test_sweep_plan_on_a_slab(lib):
    n, heads, d = 6007, 4, 64
    g = _graph(n, 5)
    q, k, v = G.make_features(n, heads, d, kind="normal", seed=2)
    Q, K, V = q.cuda(), k.cuda(), v.cuda()
    fmt = F.convert_csr_to_block_sparse(n, g.row_ptr, g.col_ind)
    full = F.fused3s_forward(Q, K, V, fmt, plan=F.make_sweep_plan(fmt, heads, d, chunk_cols=24), check_status=True)
    lo, hi = 100, 301
    order = torch.arange(lo, hi, dtype=torch.int32, device="cuda")
    plan = F.make_sweep_plan(fmt, heads, d, order=order, chunk_cols=24, window_range=(lo, hi))
    r0, r1 = 16 * lo, 16 * hi
    slab = F.fused3s_forward(Q[r0:r1].contiguous(), K, V, fmt, plan=plan, q_window_base=lo, check_status=True)
    assert torch.equal(slab, full[r0:r1])


def test_sweep_plan_hub_window(lib):
    """A hub window cut into many chunk pieces, carried in sequence."""
    n = 1 << 17
    nrw = n // 16
    c = np.arange(nrw)
    rng = np.random.default_rng(1)
    g = G.csr_from_edges(n, np.concatenate([c % 16, rng.integers(16, n, 50_000)]),
                         np.concatenate([16 * c + 3, rng.integers(0, n, 50_000)]))
    Q, K, V = G.make_features_device(n, 8, 64, "normal", seed=4)
    fmt = F.convert_csr_to_block_sparse(n, g.row_ptr, g.col_ind)
    plan = F.make_sweep_plan(fmt, 8, 64, chunk_cols=512)
    O = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True)
    off, cols = fmt.to_host()
    got, want = oracle.sampled_check(n, off, cols, np.array([0, 1, 100]), Q, K, V, O, threads=8)
    ma, rl = oracle.max_abs(got, want), oracle.rel_l2(got, want)
    assert ma <= MAX_ABS_TOL and rl <= REL_L2_TOL, f"maxabs={ma:.3e} relL2={rl:.3e}"


def test_sweep_plan_repeats_at_scale(lib):
    """Repeatability where pieces of one window meet on the same SM: the c4s
    R-MAT graph (2^18 nodes, 3.8 M blocks) in 2048-column chunks, eight
    pieces per window.  Every launch must give the same bits (a piece that
    folded in an older carried state made some launches differ), and the
    result must match the plain forward within the bar."""
    dev = torch.device("cuda")
    g = G.make_graph("c4s", device="cuda")
    n = g.num_nodes
    fmt = F.convert_csr_to_block_sparse(n, torch.from_numpy(g.row_ptr).to(dev), torch.from_numpy(g.col_ind).to(dev))
    Q, K, V = G.make_features_device(n, 8, 64, "normal", seed=42)
    plan = F.make_sweep_plan(fmt, 8, 64, chunk_cols=2048)
    first = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True)
    for _ in range(10):
        again = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True)
        assert torch.equal(again, first)
    plain = F.fused3s_forward(Q, K, V, fmt, check_status=True)
    a, b = first.cpu().numpy(), plain.cpu().numpy()
    ma, rl = oracle.max_abs(a, b), oracle.rel_l2(a, b)
    assert ma <= MAX_ABS_TOL and rl <= REL_L2_TOL, f"maxabs={ma:.3e} relL2={rl:.3e}"
