"""`torch.ops.fused3s.block_attention` and `block_attention_planned`: the
fused forward as PyTorch custom operators, for graph-transformer code that
composes it with other torch ops (torch.compile, torch.export, CUDA-graph
capture).  The operators run libfused3s.so's f3s_forward_ex on the tensors'
device and stream; their fake (meta) implementations only describe the
output, so tracing needs no GPU.

Forward only: the reference path has no backward.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import api as _api


@torch.library.custom_op("fused3s::block_attention", mutates_args=(), device_types="cuda")
def block_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, window_offsets: torch.Tensor,
                    block_cols: torch.Tensor, order: torch.Tensor, num_nodes: int, q_window_base: int = 0,
                    out_dtype: torch.dtype = torch.float32,
                    block_hints: Optional[torch.Tensor] = None) -> torch.Tensor:
    """O = block-sparse softmax(Q K^T) V over the windows in `order`.

    Q: fp16 [q_rows, H, d] (rows 16*q_window_base ...), K / V: fp16
    [num_nodes, H, d]; window_offsets / block_cols: the converter's output
    (int32); order: int32 window ids; block_hints: optional uint8 per block.
    Returns O [q_rows, H, d] of out_dtype (rows of windows not in `order` are
    left unwritten)."""
    nrw = int(window_offsets.numel()) - 1
    fmt = _api.BlockSparseFormat(nrw, window_offsets, block_cols, num_nodes)
    return _api.fused3s_forward(Q, K, V, fmt, order=order, q_window_base=q_window_base, block_hints=block_hints,
                                out_dtype=out_dtype)


# With a work plan: the plan buffer also holds the pieces' partial softmax
# states, which every call writes before reading.  The operator mutates
# `plan` and says so, so a tracer never reorders two calls that share a plan
# (no result depends on the buffer's earlier contents).
@torch.library.custom_op("fused3s::block_attention_planned", mutates_args=("plan",), device_types="cuda")
def block_attention_planned(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, window_offsets: torch.Tensor,
                            block_cols: torch.Tensor, num_nodes: int, plan: torch.Tensor, plan_max_blocks: int,
                            q_window_base: int = 0, out_dtype: torch.dtype = torch.float32,
                            block_hints: Optional[torch.Tensor] = None) -> torch.Tensor:
    """block_attention over the windows a plan lists (plan: the `.buffer` of
    make_plan, made for this H and d with piece size plan_max_blocks); heavy
    windows run as several pieces and are merged."""
    nrw = int(window_offsets.numel()) - 1
    fmt = _api.BlockSparseFormat(nrw, window_offsets, block_cols, num_nodes)
    q3 = Q if Q.dim() == 3 else Q.unsqueeze(1)
    fp = _api.ForwardPlan(plan, int(q3.shape[1]), int(q3.shape[2]), int(plan_max_blocks))
    return _api.fused3s_forward(Q, K, V, fmt, q_window_base=q_window_base, block_hints=block_hints, plan=fp,
                                out_dtype=out_dtype)


def _check_inputs(Q, K, V, window_offsets, block_cols, num_nodes):
    torch._check(Q.dtype == torch.float16 and K.dtype == torch.float16 and V.dtype == torch.float16,
                 lambda: "Q, K, V must be float16")
    torch._check(window_offsets.dtype == torch.int32 and block_cols.dtype == torch.int32,
                 lambda: "the format must be int32")
    torch._check(K.shape[0] == num_nodes, lambda: "K rows must equal num_nodes")


@block_attention.register_fake
def _(Q, K, V, window_offsets, block_cols, order, num_nodes, q_window_base=0, out_dtype=torch.float32,
      block_hints=None):
    _check_inputs(Q, K, V, window_offsets, block_cols, num_nodes)
    torch._check(order.dtype == torch.int32, lambda: "order must be int32")
    return Q.new_empty(Q.shape, dtype=out_dtype)


@block_attention_planned.register_fake
def _(Q, K, V, window_offsets, block_cols, num_nodes, plan, plan_max_blocks, q_window_base=0,
      out_dtype=torch.float32, block_hints=None):
    _check_inputs(Q, K, V, window_offsets, block_cols, num_nodes)
    torch._check(plan.dtype == torch.uint8, lambda: "plan must be a uint8 buffer")
    return Q.new_empty(Q.shape, dtype=out_dtype)
