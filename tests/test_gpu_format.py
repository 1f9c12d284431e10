"""GPU converter and window order: bit-exact against the oracle and the
golden fixtures produced by the reference's own compiled functions."""
import numpy as np
import pytest
import torch

import oracle
import fused3s_b200 as F
from fused3s_b200 import graphs as G
from fused3s_b200._lib import F3S_ERR_BAD_CSR, Fused3SError

pytestmark = pytest.mark.gpu


def gpu_convert(n, rp, ci):
    fmt = F.convert_csr_to_block_sparse(n, rp, ci)
    off, cols = fmt.to_host()
    return fmt, off, cols


def test_convert_golden_cases(lib, golden_graphs):
    for name, c in golden_graphs.items():
        n = int(c["N"][0])
        _, off, cols = gpu_convert(n, c["row_ptr"], c["col_ind"])
        assert np.array_equal(off, c["offsets"]), name
        assert np.array_equal(cols, c["cols"]), name


def test_order_golden_cases(lib, golden_graphs):
    for name, c in golden_graphs.items():
        n = int(c["N"][0])
        fmt, off, _ = gpu_convert(n, c["row_ptr"], c["col_ind"])
        order = F.generate_balanced_window_order(fmt).cpu().numpy()
        cnt = np.diff(off)
        # the block-count sequence equals the reference std::sort result
        assert np.array_equal(cnt[order], cnt[c["ref_order"]]), name
        # the permutation is the stable one (ties by ascending window id)
        assert np.array_equal(order, oracle.window_order(off)), name


def _random_csr(rng, n, m):
    s = np.sort(rng.integers(0, n, m))
    d = rng.integers(0, n, m)  # unsorted rows with duplicates
    rp = np.zeros(n + 1, np.int64)
    np.cumsum(np.bincount(s, minlength=n), out=rp[1:])
    return rp.astype(np.int32), d.astype(np.int32)


@pytest.mark.parametrize("n", [1, 15, 16, 17, 33, 1000, 4097, 70001])
def test_convert_random_unsorted_duplicates(lib, n):
    rng = np.random.default_rng(n)
    rp, ci = _random_csr(rng, n, 5 * n)
    _, off, cols = gpu_convert(n, rp, ci)
    eo, ec = oracle.convert(n, rp, ci)
    assert np.array_equal(off, eo) and np.array_equal(cols, ec)


def test_convert_no_edges(lib):
    n = 100
    rp = np.zeros(n + 1, np.int32)
    _, off, cols = gpu_convert(n, rp, np.zeros(0, np.int32))
    assert np.array_equal(off, np.zeros(8, np.int32)) and cols.size == 0


def test_convert_heavy_windows(lib):
    """Windows above the shared-memory sort capacity take the bitmap path."""
    rng = np.random.default_rng(5)
    n = 200_000
    deg = np.full(n, 2)
    deg[:16] = 3000          # window 0: 48k edges
    deg[32:48] = 300         # window 2: 4800 edges, just over the 4096 cap
    deg[4096 * 16] = 5000    # a lone hub
    rp = np.zeros(n + 1, np.int64)
    np.cumsum(deg, out=rp[1:])
    ci = rng.integers(0, n, int(rp[-1])).astype(np.int32)
    _, off, cols = gpu_convert(n, rp.astype(np.int32), ci)
    eo, ec = oracle.convert(n, rp.astype(np.int32), ci)
    assert np.array_equal(off, eo) and np.array_equal(cols, ec)


def test_convert_bitmap_two_passes(lib):
    """nrw > 2^20 block columns: the heavy-window bitmap runs in two passes."""
    n = (1 << 24) + 37
    rng = np.random.default_rng(9)
    deg = np.zeros(n, np.int64)
    deg[5] = 6000                      # one heavy window spanning the whole id range
    deg[rng.integers(16, n, 2000)] += 1
    rp = np.zeros(n + 1, np.int64)
    np.cumsum(deg, out=rp[1:])
    ci = rng.integers(0, n, int(rp[-1])).astype(np.int32)
    ci[:10] = n - 1                    # last block column
    _, off, cols = gpu_convert(n, rp.astype(np.int32), ci)
    eo, ec = oracle.convert(n, rp.astype(np.int32), ci)
    assert np.array_equal(off, eo) and np.array_equal(cols, ec)


@pytest.mark.parametrize("config", ["c1", "c2", "c3"])
def test_convert_configs(lib, config):
    g = G.make_graph(config)
    _, off, cols = gpu_convert(g.num_nodes, g.row_ptr, g.col_ind)
    eo, ec = oracle.convert(g.num_nodes, g.row_ptr, g.col_ind)
    assert np.array_equal(off, eo) and np.array_equal(cols, ec)


def test_convert_c4_rmat(lib):
    g = G.make_graph("c4", device="cuda")
    fmt, off, cols = gpu_convert(g.num_nodes, g.row_ptr, g.col_ind)
    eo, ec = oracle.convert(g.num_nodes, g.row_ptr, g.col_ind)
    assert np.array_equal(off, eo) and np.array_equal(cols, ec)
    order = F.generate_balanced_window_order(fmt).cpu().numpy()
    assert np.array_equal(order, oracle.window_order(off))


@pytest.mark.parametrize("nrw", [1, 255, 256, 257, 2048, 65536, 300_001])
def test_order_arbitrary_counts(lib, nrw):
    rng = np.random.default_rng(nrw)
    cnt = np.minimum(rng.zipf(1.6, nrw), nrw).astype(np.int64)
    cnt[rng.integers(0, nrw, nrw // 10 + 1)] = 0
    off = np.zeros(nrw + 1, np.int64)
    np.cumsum(cnt, out=off[1:])
    fmt = F.BlockSparseFormat(nrw, torch.from_numpy(off.astype(np.int32)).cuda(),
                              torch.zeros(1, dtype=torch.int32, device="cuda"), nrw * 16)
    order = F.generate_balanced_window_order(fmt).cpu().numpy()
    assert np.array_equal(order, np.argsort(-cnt, kind="stable"))


def test_convert_rejects_bad_csr(lib):
    n = 40
    rp = np.arange(0, 2 * n + 1, 2, dtype=np.int32)
    ci = np.zeros(2 * n, np.int32)
    ci[7] = n  # column out of range
    with pytest.raises(Fused3SError) as e:
        F.convert_csr_to_block_sparse(n, rp, ci)
    assert e.value.status == F3S_ERR_BAD_CSR
    ci[7] = 0
    rp2 = rp.copy()
    rp2[5] = rp2[6] + 1  # decreasing row_ptr
    with pytest.raises(Fused3SError) as e:
        F.convert_csr_to_block_sparse(n, rp2, ci)
    assert e.value.status == F3S_ERR_BAD_CSR
    # the device is still healthy: a valid call succeeds afterwards
    _, off, cols = gpu_convert(n, rp, ci)
    eo, ec = oracle.convert(n, rp, ci)
    assert np.array_equal(off, eo) and np.array_equal(cols, ec)
