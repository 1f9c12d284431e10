"""The custom operator torch.ops.fused3s.block_attention: its schema and fake
implementation on CPU (meta tensors, no GPU), and on the GPU the same result
as fused3s_forward plus torch.library.opcheck."""
import numpy as np
import pytest
import torch

import fused3s_b200 as F
from fused3s_b200 import graphs as G


def test_op_is_registered_with_a_fake_impl():
    op = torch.ops.fused3s.block_attention
    assert "block_attention" in str(op.default._schema)
    n, h, d = 100, 2, 64
    m = torch.device("meta")
    Q = torch.empty(n, h, d, dtype=torch.float16, device=m)
    off = torch.empty(8, dtype=torch.int32, device=m)
    cols = torch.empty(20, dtype=torch.int32, device=m)
    order = torch.empty(7, dtype=torch.int32, device=m)
    out = op(Q, Q, Q, off, cols, order, n, 0, torch.bfloat16)
    assert out.shape == (n, h, d) and out.dtype == torch.bfloat16 and out.device.type == "meta"
    with pytest.raises(Exception):
        op(Q.float(), Q, Q, off, cols, order, n)


@pytest.mark.gpu
def test_op_matches_fused3s_forward(lib):
    g = G.powerlaw_graph(num_nodes=1500, directed_edges=12000, max_degree=300, seed=4)
    q, k, v = (t.cuda() for t in G.make_features(g.num_nodes, 2, 64, kind="normal", seed=3))
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    order = F.generate_balanced_window_order(fmt)
    ref = F.fused3s_forward(q, k, v, fmt, order=order)
    op = torch.ops.fused3s.block_attention
    got = op(q, k, v, fmt.window_offsets, fmt.block_col_indices, order, g.num_nodes)
    assert torch.equal(got, ref)
    plan = F.make_plan(fmt, 2, 64, order=order, max_blocks=6)
    ref_p = F.fused3s_forward(q, k, v, fmt, plan=plan, out_dtype=torch.float16)
    opp = torch.ops.fused3s.block_attention_planned
    got_p = opp(q, k, v, fmt.window_offsets, fmt.block_col_indices, g.num_nodes, plan.buffer, plan.max_blocks, 0,
                torch.float16)
    assert torch.equal(got_p, ref_p)
    torch.library.opcheck(op, (q, k, v, fmt.window_offsets, fmt.block_col_indices, order, g.num_nodes),
                          test_utils=("test_schema", "test_faketensor"))
    # the plan buffer is declared mutated (its partial states are written)
    torch.library.opcheck(opp, (q, k, v, fmt.window_offsets, fmt.block_col_indices, g.num_nodes, plan.buffer,
                                plan.max_blocks), test_utils=("test_schema", "test_faketensor"))


def test_ops_declare_what_they_mutate():
    def mutated(op):
        return [a.name for a in op.default._schema.arguments if a.alias_info is not None and a.alias_info.is_write]

    assert mutated(torch.ops.fused3s.block_attention) == []
    assert mutated(torch.ops.fused3s.block_attention_planned) == ["plan"]
