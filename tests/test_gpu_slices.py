"""K / V held in slices of block columns (f3s_forward_pieces + f3s_plan_merge):
the single-GPU form of the ring that passes K / V slices between GPUs.

Each slice's pieces run against a buffer holding only that slice's K / V
rows; the split windows are merged once at the end.  The result must match
the oracle within the fused kernel's bar, be bit-identical whatever order
the slices arrive in (every rank of a ring sees them in a different order),
and equal the same plan run against the whole K / V.
"""
import numpy as np
import pytest
import torch

import oracle
import fused3s_b200 as F
from conftest import MAX_ABS_TOL, REL_L2_TOL
from fused3s_b200 import _lib
from fused3s_b200 import graphs as G

pytestmark = pytest.mark.gpu


def _setup(n, heads, d, seed):
    g = G.powerlaw_graph(num_nodes=n, directed_edges=8 * n, max_degree=400, seed=seed)
    q, k, v = G.make_features(g.num_nodes, heads, d, kind="normal", seed=seed)
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    return g, fmt, q.cuda(), k.cuda(), v.cuda(), (q, k, v)


def _sliced_forward(fmt, plan, cuts, rows, Q, K, V, slice_order, out_dtype=torch.float32):
    O = torch.full(Q.shape, float("nan"), dtype=out_dtype, device=Q.device)
    for j in slice_order:
        r0, r1 = rows[j]
        Ks, Vs = K[r0:r1].clone(), V[r0:r1].clone()  # only this slice's rows exist
        a, b = plan.piece_ranges[j]
        F.forward_pieces(Q, Ks, Vs, fmt, plan, O, piece_begin=a, piece_end=b, kv_col_base=int(cuts[j]),
                         check_status=True)
    F.plan_merge(plan, O, fmt.num_nodes)
    torch.cuda.synchronize()
    return O


@pytest.mark.parametrize("n,heads,d,parts", [(3001, 4, 64, 3), (2051, 2, 128, 2), (4096, 8, 64, 8)])
def test_sliced_kv_matches_oracle_in_any_slice_order(lib, n, heads, d, parts):
    g, fmt, Q, K, V, host = _setup(n, heads, d, seed=n)
    cuts, rows = F.column_slices(g.num_nodes, parts)
    plan = F.make_sliced_plan(fmt, heads, d, cuts)
    O1 = _sliced_forward(fmt, plan, cuts, rows, Q, K, V, range(parts))
    O2 = _sliced_forward(fmt, plan, cuts, rows, Q, K, V, reversed(range(parts)))
    assert torch.equal(O1, O2)
    # the same plan against the whole K / V: bit-identical
    O3 = torch.full(Q.shape, float("nan"), dtype=torch.float32, device=Q.device)
    F.forward_pieces(Q, K, V, fmt, plan, O3, check_status=True)
    F.plan_merge(plan, O3, fmt.num_nodes)
    assert torch.equal(O1, O3)
    off, cols = fmt.to_host()
    q, k, v = (x.float().numpy() for x in host)
    ref = oracle.block_attention(g.num_nodes, q, k, v, off, cols, threads=8)
    o = O1.cpu().numpy()
    ma, rl = oracle.max_abs(o, ref), oracle.rel_l2(o, ref)
    assert ma <= MAX_ABS_TOL and rl <= REL_L2_TOL, f"maxabs={ma:.3e} relL2={rl:.3e}"


def test_sliced_kv_half_output(lib):
    g, fmt, Q, K, V, _ = _setup(3001, 4, 64, seed=9)
    cuts, rows = F.column_slices(g.num_nodes, 4)
    plan = F.make_sliced_plan(fmt, 4, 64, cuts)
    O32 = _sliced_forward(fmt, plan, cuts, rows, Q, K, V, [1, 3, 0, 2])
    O16 = _sliced_forward(fmt, plan, cuts, rows, Q, K, V, [3, 2, 1, 0], out_dtype=torch.float16)
    assert torch.equal(O16, O32.to(torch.float16))


def test_block_outside_the_held_slice_is_reported(lib):
    g, fmt, Q, K, V, _ = _setup(3001, 2, 64, seed=4)
    cuts, rows = F.column_slices(g.num_nodes, 3)
    plan = F.make_sliced_plan(fmt, 2, 64, cuts)
    O = torch.zeros(Q.shape, dtype=torch.float32, device=Q.device)
    a, b = plan.piece_ranges[0]
    r0, r1 = rows[1]
    with pytest.raises(_lib.Fused3SError) as e:  # slice 0's pieces against slice 1's rows
        F.forward_pieces(Q, K[r0:r1].clone(), V[r0:r1].clone(), fmt, plan, O, piece_begin=a, piece_end=b,
                         kv_col_base=int(cuts[1]), check_status=True)
    assert e.value.status == _lib.F3S_ERR_BAD_FORMAT
    # the context still works: the right slice afterwards is fine
    r0, r1 = rows[0]
    F.forward_pieces(Q, K[r0:r1].clone(), V[r0:r1].clone(), fmt, plan, O, piece_begin=a, piece_end=b,
                     kv_col_base=0, check_status=True)


def test_piece_range_and_slice_arguments_are_validated(lib):
    g, fmt, Q, K, V, _ = _setup(1000, 1, 64, seed=2)
    cuts, rows = F.column_slices(g.num_nodes, 2)
    plan = F.make_sliced_plan(fmt, 1, 64, cuts)
    O = torch.zeros(Q.shape, dtype=torch.float32, device=Q.device)
    # a slice that stops inside the graph must end on a block-column boundary
    with pytest.raises(_lib.Fused3SError) as e:
        F.forward_pieces(Q, K[:100], V[:100], fmt, plan, O, kv_col_base=0)
    assert e.value.status == _lib.F3S_ERR_INVALID_VALUE
    # and must lie inside the graph
    with pytest.raises(_lib.Fused3SError):
        F.forward_pieces(Q, K[:512], V[:512], fmt, plan, O, kv_col_base=40)
    # a piece range beyond the plan is reported by the kernel
    with pytest.raises(_lib.Fused3SError) as e:
        F.forward_pieces(Q, K, V, fmt, plan, O, piece_begin=0, piece_end=10**6, check_status=True)
    assert e.value.status == _lib.F3S_ERR_BAD_FORMAT
