"""The largest configuration, C5, at its real size: R-MAT 2^24 nodes, average
degree 32 (~537M directed edges), H=4, d=128, fp16 Q/K/V ~ N(0,1)/sqrt(d).

This is the regime where the reference's int32 index arithmetic would
overflow (window * 16 * feat_dim, src/fused3s_v2.cu:111,127,161,222,244)
and where K and V span 17 GB each, so the TMA maps address well beyond
2^32 bytes.  Checked against the oracle (the C restatement, pinned to the
reference's own functions):
  * the converter output, bit for bit, over the whole graph;
  * the window order (the stable order exactly; the reference's block-count
    sequence when the compiled reference is present);
  * the fused output of the bench's configuration (automatic plan, L2
    hints) on 128 seeded random windows x all heads against the reference's
    float32 CPU function, and on the 3 heaviest windows (hub windows of
    several hundred thousand blocks) x the first and last head against the
    same block semantics in float64 (the float32 reference's softmax sum
    drifts over millions of columns), at max-abs 2e-2 / rel-L2 1e-3.
About 90 GB of device memory and a few minutes of host time.
"""
import os

import numpy as np
import pytest
import torch

import oracle
import fused3s_b200 as F
from conftest import MAX_ABS_TOL, REL_L2_TOL
from fused3s_b200 import graphs as G

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


@pytest.fixture(scope="module")
def c5():
    cfg = G.CONFIGS["c5"]
    g = G.make_graph("c5", device="cuda")
    rp = torch.from_numpy(g.row_ptr).cuda()
    ci = torch.from_numpy(g.col_ind).cuda()
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, rp, ci)
    del rp, ci
    torch.cuda.empty_cache()
    return g, cfg, fmt


def test_c5_converter_and_order_bit_exact(lib, c5):
    g, cfg, fmt = c5
    off, cols = fmt.to_host()
    want_off, want_cols = oracle.convert(g.num_nodes, g.row_ptr, g.col_ind, threads=THREADS)
    assert np.array_equal(off, want_off)
    assert np.array_equal(cols, want_cols)
    assert off[-1] > 2**28  # hundreds of millions of active blocks
    order = F.generate_balanced_window_order(fmt).cpu().numpy()
    assert np.array_equal(order, oracle.window_order(off))
    if oracle.ref_available():
        cnt = np.diff(off)
        assert np.array_equal(cnt[order], cnt[oracle.ref_window_order(off)])


def test_c5_fused_output_sampled(lib, c5):
    g, cfg, fmt = c5
    H, d = cfg.heads, cfg.head_dim
    N = g.num_nodes
    Q, K, V = G.make_features_device(N, H, d, cfg.features, seed=42)
    order = F.generate_balanced_window_order(fmt)
    plan = F.make_plan(fmt, H, d, order=order)
    hints = F.block_hints(fmt, H, d, order=order)
    O = F.fused3s_forward(Q, K, V, fmt, plan=plan, block_hints=hints, check_status=True)
    torch.cuda.synchronize()
    off = fmt.window_offsets.cpu().numpy()
    cols = fmt.block_col_indices.cpu().numpy()
    cnt = np.diff(off)
    rng = np.random.default_rng(5)
    rand = np.unique(rng.choice(len(cnt), 128, replace=False))
    got, want = oracle.sampled_check(N, off, cols, rand, Q, K, V, O, threads=THREADS)
    ma, rl = oracle.max_abs(got, want), oracle.rel_l2(got, want)
    assert ma <= MAX_ABS_TOL and rl <= REL_L2_TOL, f"random windows: maxabs={ma:.3e} relL2={rl:.3e}"
    # The 3 heaviest windows hold several hundred thousand blocks (millions
    # of columns per row).  There the reference's float32 softmax sum, added
    # column by column, drifts (its adds round to the accumulator's ulp), so
    # the yardstick is the same block semantics in float64
    # (oracle.block_attention_exact); the float32 reference's own distance
    # from it is reported beside ours.
    heavy = np.sort(np.argsort(-cnt, kind="stable")[:3])
    got, ref32 = oracle.sampled_check(N, off, cols, heavy, Q, K, V, O, heads=[0, H - 1], threads=THREADS)
    exact = []
    for w in heavy:
        rows = torch.arange(16 * w, min(16 * w + 16, N), device=Q.device)
        exact.append(np.stack([oracle.block_attention_exact(N, Q[rows, h, :].float().cpu().numpy(), K[:, h, :],
                                                            V[:, h, :], off, cols, int(w))
                               for h in (0, H - 1)], axis=1))
    exact = np.concatenate(exact)
    ma, rl = oracle.max_abs(got, exact), oracle.rel_l2(got, exact)
    print(f"heaviest windows {cnt[heavy].tolist()} blocks: fused vs float64 maxabs={ma:.3e} relL2={rl:.3e}; "
          f"float32 reference vs float64 maxabs={oracle.max_abs(ref32, exact):.3e} "
          f"relL2={oracle.rel_l2(ref32, exact):.3e}")
    assert ma <= MAX_ABS_TOL and rl <= REL_L2_TOL, f"heaviest windows: maxabs={ma:.3e} relL2={rl:.3e}"
    # and within the max-abs bar of the float32 reference itself
    assert oracle.max_abs(got, ref32) <= MAX_ABS_TOL
