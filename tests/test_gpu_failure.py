"""Failure detection without a GPU fault: every device-side wait is bounded,
and errors come back as status codes while the context stays usable."""
import numpy as np
import pytest
import torch

import fused3s_b200 as F
from fused3s_b200 import _lib
from fused3s_b200 import graphs as G

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports(lib):
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.f3s_selftest_wait_timeout(2_000_000, ws.data_ptr(), 256, stream) == 0  # 2 ms bound
    assert lib.f3s_workspace_status(ws.data_ptr(), stream) == _lib.F3S_ERR_TIMEOUT
    # status is cleared once read, and the context still works
    assert lib.f3s_workspace_status(ws.data_ptr(), stream) == 0
    x = torch.arange(10, device="cuda").sum().item()
    assert x == 45


def test_window_id_outside_slab_is_reported(lib):
    g = G.make_graph("c1")
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    q, k, v = (t.cuda() for t in G.make_features(g.num_nodes, 1, 64))
    bad = torch.tensor([0, fmt.num_row_windows + 5], dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.Fused3SError) as e:
        F.fused3s_forward(q, k, v, fmt, order=bad, check_status=True)
    assert e.value.status == _lib.F3S_ERR_BAD_FORMAT
    # a correct call right after succeeds
    F.fused3s_forward(q, k, v, fmt, check_status=True)


def test_unsupported_head_dim_rejected_on_host(lib):
    g = G.make_graph("c1")
    fmt = F.convert_csr_to_block_sparse(g.num_nodes, g.row_ptr, g.col_ind)
    q = torch.zeros(g.num_nodes, 1, 96, dtype=torch.float16, device="cuda")
    with pytest.raises(_lib.Fused3SError) as e:
        F.fused3s_forward(q, q, q, fmt)
    assert e.value.status == _lib.F3S_ERR_UNSUPPORTED


def test_workspace_too_small_rejected(lib):
    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    rp = torch.zeros(101, dtype=torch.int32, device="cuda")
    off = torch.zeros(8, dtype=torch.int32, device="cuda")
    st = lib.f3s_convert(rp.data_ptr(), None, 100, 0, off.data_ptr(), None, ws.data_ptr(), 16, None, stream)
    assert st == _lib.F3S_ERR_WORKSPACE
