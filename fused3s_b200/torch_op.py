"""`torch.ops.fused3s.block_attention`: the fused forward as a PyTorch custom
operator, for graph-transformer code that composes it with other torch ops
(torch.compile, torch.export, CUDA-graph capture).  The operator runs
libfused3s.so's f3s_forward_ex on the tensors' device and stream; its fake
(meta) implementation only describes the output, so tracing needs no GPU.

Forward only: the reference path has no backward.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import api as _api


# The plan buffer also holds the pieces' partial softmax states: scratch that
# every call overwrites before reading, so no result depends on its earlier
# contents (calls sharing one plan must still run one at a time, as on one
# stream).
@torch.library.custom_op("fused3s::block_attention", mutates_args=(), device_types="cuda")
def block_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, window_offsets: torch.Tensor,
                    block_cols: torch.Tensor, order: torch.Tensor, num_nodes: int, q_window_base: int = 0,
                    out_dtype: torch.dtype = torch.float32, block_hints: Optional[torch.Tensor] = None,
                    plan: Optional[torch.Tensor] = None, plan_max_blocks: int = 0) -> torch.Tensor:
    """O = block-sparse softmax(Q K^T) V over the windows in `order`.

    Q: fp16 [q_rows, H, d] (rows 16*q_window_base ...), K / V: fp16
    [num_nodes, H, d]; window_offsets / block_cols: the converter's output
    (int32); order: int32 window ids; block_hints: optional uint8 per block;
    plan: optional plan buffer from make_plan (its `.buffer`), made for this
    H and d with piece size plan_max_blocks.  Returns O [q_rows, H, d] of
    out_dtype (rows of windows not in `order` are left unwritten)."""
    nrw = int(window_offsets.numel()) - 1
    fmt = _api.BlockSparseFormat(nrw, window_offsets, block_cols, num_nodes)
    fp = None
    if plan is not None:
        q3 = Q if Q.dim() == 3 else Q.unsqueeze(1)
        fp = _api.ForwardPlan(plan, int(q3.shape[1]), int(q3.shape[2]), int(plan_max_blocks))
    return _api.fused3s_forward(Q, K, V, fmt, order=order, q_window_base=q_window_base, block_hints=block_hints,
                                plan=fp, out_dtype=out_dtype)


@block_attention.register_fake
def _(Q, K, V, window_offsets, block_cols, order, num_nodes, q_window_base=0, out_dtype=torch.float32,
      block_hints=None, plan=None, plan_max_blocks=0):
    torch._check(Q.dtype == torch.float16 and K.dtype == torch.float16 and V.dtype == torch.float16,
                 lambda: "Q, K, V must be float16")
    torch._check(window_offsets.dtype == torch.int32 and block_cols.dtype == torch.int32
                 and order.dtype == torch.int32, lambda: "format and order must be int32")
    torch._check(K.shape[0] == num_nodes, lambda: "K rows must equal num_nodes")
    return Q.new_empty(Q.shape, dtype=out_dtype)
