"""CSR text decoded on the GPU (f3s_parse_int32, load_csr_graph_device):
exact against numpy on random texts with every separator the reference's
`>>` reader accepts, numbers across thread and tile boundaries, int32
limits, and the error cases; a dataset directory read on the device equals
the host reader and converts to the same format."""
import numpy as np
import pytest
import torch

import fused3s_b200 as F
from fused3s_b200 import _lib
from fused3s_b200 import graphs as G

pytestmark = pytest.mark.gpu


def _format(values, rng):
    seps = [" ", "\n", "\t", "\r\n", "  ", " \n "]
    out = [rng.choice(["", " ", "\n"])]
    for v in values:
        out.append(str(int(v)))
        out.append(seps[rng.integers(len(seps))])
    return "".join(out).encode()


@pytest.mark.parametrize("n", [0, 1, 7, 1000, 100_003])
def test_parse_random_texts(lib, n):
    rng = np.random.default_rng(n)
    v = rng.integers(-(2**31), 2**31, n, dtype=np.int64)
    v[: min(n, 4)] = [2**31 - 1, -(2**31), 0, 7][: min(n, 4)]
    small = rng.random(n) < 0.5
    v[small] = rng.integers(0, 100, small.sum())
    got = F.parse_int32_text(_format(v, rng)).cpu().numpy()
    assert np.array_equal(got, v.astype(np.int32))


def test_parse_long_numbers_across_tiles(lib):
    # 10-digit numbers with single separators: every 16-byte thread span and
    # 4096-byte tile boundary falls inside some number
    v = np.arange(1_000_000_000, 1_000_000_000 + 50_000, 37, dtype=np.int64)
    text = (" ".join(str(x) for x in v)).encode()
    assert np.array_equal(F.parse_int32_text(text).cpu().numpy(), v.astype(np.int32))


@pytest.mark.parametrize("text,status", [(b"1 2 x 3", _lib.F3S_ERR_INVALID_VALUE), (b"12-3", _lib.F3S_ERR_INVALID_VALUE),
                                         (b"5 - 6", _lib.F3S_ERR_INVALID_VALUE), (b"2147483648", _lib.F3S_ERR_TOO_LARGE),
                                         (b"-2147483649", _lib.F3S_ERR_TOO_LARGE),
                                         (b"123456789012", _lib.F3S_ERR_TOO_LARGE)])
def test_parse_errors(lib, text, status):
    with pytest.raises(_lib.Fused3SError) as e:
        F.parse_int32_text(text)
    assert e.value.status == status
    assert np.array_equal(F.parse_int32_text(b"4 5\n6").cpu().numpy(), [4, 5, 6])  # device still fine


def test_parse_more_numbers_than_room(lib):
    with pytest.raises(_lib.Fused3SError) as e:
        F.parse_int32_text(b"1 2 3 4", max_count=3)
    assert e.value.status == _lib.F3S_ERR_WORKSPACE


def test_load_csr_graph_device_equals_host_reader(lib, tmp_path):
    g = G.make_graph("c2")
    d = tmp_path / "c2"
    d.mkdir()
    (d / "meta.txt").write_text(f"{g.num_nodes} {g.num_edges}\n")
    np.savetxt(d / "row_ptr.txt", g.row_ptr, fmt="%d")
    np.savetxt(d / "col_idx.txt", g.col_ind, fmt="%d")
    host = F.load_csr_graph(str(d))
    dev = F.load_csr_graph_device(str(d))
    assert dev.row_ptr.is_cuda and dev.col_ind.is_cuda
    assert np.array_equal(dev.row_ptr.cpu().numpy(), host.row_ptr)
    assert np.array_equal(dev.col_ind.cpu().numpy(), host.col_ind)
    a = F.convert_csr_to_block_sparse(dev.num_nodes, dev.row_ptr, dev.col_ind).to_host()
    b = F.convert_csr_to_block_sparse(host.num_nodes, host.row_ptr, host.col_ind).to_host()
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
