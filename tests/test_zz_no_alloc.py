"""f3s_convert_noalloc: the converter for callers that cannot allocate device
memory (a plugin inside a framework whose allocator already holds the GPU's
memory, or a service that never calls cudaMalloc / cudaFree after start-up).
Its scratch is a fixed 32 MiB array inside the library.

Called through the C ABI and checked against the existing entry point
(f3s_convert, through the Python API) and against the oracle's restatement
of the reference converter -- integer output, so bit for bit --
on two calls in a row, the second on a smaller graph so that anything the
first call left in the shared array would show.  This file is collected
last so that a run stopping at the first failure has run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import fused3s_b200 as F
import oracle
from fused3s_b200 import _lib
from fused3s_b200 import graphs as G

pytestmark = pytest.mark.gpu


def convert_noalloc(lib, n, row_ptr, col_ind):
    rp = torch.from_numpy(np.ascontiguousarray(row_ptr, np.int32)).cuda()
    ci = torch.from_numpy(np.ascontiguousarray(col_ind, np.int32)).cuda()
    nnz = int(ci.numel())
    nrw = (n + 15) // 16
    off = torch.full((nrw + 1,), -7, dtype=torch.int32, device="cuda")
    cols = torch.full((max(nnz, 1),), -7, dtype=torch.int32, device="cuda")
    nb = ctypes.c_int64(-1)
    st = lib.f3s_convert_noalloc(rp.data_ptr(), ci.data_ptr(), n, nnz, off.data_ptr(), cols.data_ptr(),
                                 ctypes.byref(nb), torch.cuda.current_stream().cuda_stream)
    return st, off.cpu().numpy(), cols[: max(nb.value, 0)].cpu().numpy()


def graph_with_heavy_window(seed):
    """Unsorted rows, duplicate edges, one window above the 4096-edge
    shared-memory sort (bitmap path) and a partial last window."""
    rng = np.random.default_rng(seed)
    n = 40_003
    deg = rng.integers(0, 6, n)
    deg[16:32] = 400  # window 1: 6400 edges
    rp = np.zeros(n + 1, np.int64)
    np.cumsum(deg, out=rp[1:])
    ci = rng.integers(0, n, int(rp[-1]))
    return n, rp.astype(np.int32), ci.astype(np.int32)


def test_noalloc_convert_matches_f3s_convert_twice(lib):
    big = graph_with_heavy_window(1)
    c1 = G.make_graph("c1")
    small = (c1.num_nodes, c1.row_ptr, c1.col_ind)
    for n, rp, ci in (big, small):  # two calls in a row
        st, off, cols = convert_noalloc(lib, n, rp, ci)
        assert st == _lib.F3S_SUCCESS, _lib.status_string(st)
        want = F.convert_csr_to_block_sparse(n, rp, ci)
        want_off, want_cols = want.to_host()
        assert np.array_equal(off, want_off)
        assert np.array_equal(cols, want_cols)
        # and the reference's converter, restated (bit for bit)
        ref_off, ref_cols = oracle.convert(n, rp, ci)
        assert np.array_equal(off, ref_off)
        assert np.array_equal(cols, ref_cols)


def test_noalloc_convert_limits_and_errors(lib):
    stream = torch.cuda.current_stream().cuda_stream
    rp = torch.zeros(2, dtype=torch.int32, device="cuda")
    buf = torch.zeros(16, dtype=torch.int32, device="cuda")
    nb = ctypes.c_int64(0)
    # beyond the fixed scratch: rejected before anything runs
    st = lib.f3s_convert_noalloc(rp.data_ptr(), buf.data_ptr(), 1, 9_000_000, buf.data_ptr(), buf.data_ptr(),
                                 ctypes.byref(nb), stream)
    assert st == _lib.F3S_ERR_WORKSPACE
    # the host count pointer is required (the call reports through it)
    st = lib.f3s_convert_noalloc(rp.data_ptr(), buf.data_ptr(), 1, 1, buf.data_ptr(), buf.data_ptr(), None, stream)
    assert st == _lib.F3S_ERR_INVALID_VALUE
    # a bad CSR is reported, and the next call starts clean
    n = 20
    rp_h = np.arange(0, 2 * n + 1, 2, dtype=np.int32)
    ci_h = np.zeros(2 * n, np.int32)
    ci_h[3] = n + 100
    st, _, _ = convert_noalloc(lib, n, rp_h, ci_h)
    assert st == _lib.F3S_ERR_BAD_CSR
    ci_h[3] = 5
    st, off, cols = convert_noalloc(lib, n, rp_h, ci_h)
    assert st == _lib.F3S_SUCCESS
    want_off, want_cols = F.convert_csr_to_block_sparse(n, rp_h, ci_h).to_host()
    assert np.array_equal(off, want_off) and np.array_equal(cols, want_cols)
