"""A hub row window: 16 rows whose edges reach every block column of a
graph of 2^21 nodes (131,072 active blocks in one window, H=8, d=64, so one
consumer warp accumulates every block of a head).

The tensor cores accumulate P.V into fp32 with truncation, so a single
accumulator fed ~10^5 blocks drifts toward zero; the window's O is an
average over 2 million columns and so is small, and the drift shows in the
relative error.  Work plans cut such windows into pieces of at most
MAX_PIECE_BLOCKS blocks, merged with round-to-nearest fp32 arithmetic: the
planned forward (the bench's path) must meet the parity bar on the hub
window.  The unplanned forward's error is reported for comparison."""
import numpy as np
import pytest
import torch

import oracle
import fused3s_b200 as F
from conftest import MAX_ABS_TOL, REL_L2_TOL
from fused3s_b200 import graphs as G

pytestmark = pytest.mark.gpu


def test_hub_window_meets_the_bar_with_automatic_pieces(lib):
    n, H, d = 1 << 21, 8, 64
    nrw = n // 16
    rng = np.random.default_rng(8)
    c = np.arange(nrw)
    src = np.concatenate([c % 16, rng.integers(16, n, 200_000)])  # the hub window + light noise elsewhere
    dst = np.concatenate([16 * c + (7 * c) % 16, rng.integers(0, n, 200_000)])
    g = G.csr_from_edges(n, src, dst)
    fmt = F.convert_csr_to_block_sparse(n, g.row_ptr, g.col_ind)
    off, cols = fmt.to_host()
    assert off[1] - off[0] == nrw  # every block column
    Q, K, V = G.make_features_device(n, H, d, "normal", seed=3)
    plan = F.make_plan(fmt, H, d)
    assert plan.max_blocks <= F.api.MAX_PIECE_BLOCKS
    O_plan = F.fused3s_forward(Q, K, V, fmt, plan=plan, check_status=True)
    O_whole = F.fused3s_forward(Q, K, V, fmt, check_status=True)
    torch.cuda.synchronize()
    win = np.array([0])
    got, want = oracle.sampled_check(n, off, cols, win, Q, K, V, O_plan, heads=[0, 5], threads=8)
    ma, rl = oracle.max_abs(got, want), oracle.rel_l2(got, want)
    got_w = O_whole[:16][:, [0, 5], :].float().cpu().numpy()
    print(f"hub window: planned maxabs={ma:.3e} relL2={rl:.3e}; one accumulator "
          f"maxabs={oracle.max_abs(got_w, want):.3e} relL2={oracle.rel_l2(got_w, want):.3e}")
    assert ma <= MAX_ABS_TOL and rl <= REL_L2_TOL, f"maxabs={ma:.3e} relL2={rl:.3e}"
