"""fused3s_b200 -- a B200-native (sm_100a) fused 3S engine.

CSR -> 16x16 block-sparse row windows -> descending-workload window order ->
fused SDDMM + online softmax + SpMM -> fp32 O, all on the GPU, behind the
C ABI of libfused3s.so (include/fused3s.h) and the reference-shaped host API
below.
"""
from .api import (
    BlockSparseFormat,
    GraphData,
    ForwardPlan,
    Fused3SError,
    auto_piece_blocks,
    block_hints,
    convert_csr_to_block_sparse,
    f3s_1tb1rw_kernel,
    float2half,
    forward_workspace,
    fused3s_forward,
    generate_balanced_window_order,
    load_csr_graph,
    load_csr_graph_device,
    column_chunk_pieces,
    column_slices,
    forward_pieces,
    load_plan,
    locality_order,
    make_chunked_plan,
    make_sliced_plan,
    make_sweep_plan,
    plan_merge,
    set_forward_sm_limit,
    make_plan,
    parse_int32_text,
    workspace_status,
)
from . import torch_op  # registers torch.ops.fused3s.block_attention

__all__ = [
    "BlockSparseFormat",
    "GraphData",
    "ForwardPlan",
    "Fused3SError",
    "auto_piece_blocks",
    "block_hints",
    "convert_csr_to_block_sparse",
    "f3s_1tb1rw_kernel",
    "make_plan",
    "make_chunked_plan",
    "column_chunk_pieces",
    "column_slices",
    "forward_pieces",
    "load_plan",
    "locality_order",
    "make_sliced_plan",
    "make_sweep_plan",
    "plan_merge",
    "set_forward_sm_limit",
    "float2half",
    "forward_workspace",
    "fused3s_forward",
    "generate_balanced_window_order",
    "load_csr_graph",
    "load_csr_graph_device",
    "parse_int32_text",
    "workspace_status",
]
