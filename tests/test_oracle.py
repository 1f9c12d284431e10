"""The oracle is pinned before it is trusted (CPU only).

  * the C restatement (oracle/f3s_oracle.c) reproduces the golden fixtures
    that the reference's own compiled functions produced (tests/golden/);
  * when the reference tree is present, the restatement is also compared
    live with the compiled reference on fresh random graphs, and the
    reference's vendored Cora / Citeseer CSR is checked against the committed
    digests.
"""
import hashlib
import json

import numpy as np
import pytest

import oracle
from conftest import GOLDEN
from fused3s_b200 import graphs as G

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="reference not compiled (oracle/_ref)")


def test_port_convert_matches_golden(golden_graphs):
    for name, c in golden_graphs.items():
        off, cols = oracle.convert(int(c["N"][0]), c["row_ptr"], c["col_ind"])
        assert np.array_equal(off, c["offsets"]), name
        assert np.array_equal(cols, c["cols"]), name


def test_port_order_matches_golden_keys(golden_graphs):
    """Block counts along the order equal the reference's std::sort result;
    the permutation is the stable one (ties by ascending window id)."""
    for name, c in golden_graphs.items():
        cnt = np.diff(c["offsets"])
        order = oracle.window_order(c["offsets"])
        assert np.array_equal(cnt[order], cnt[c["ref_order"]]), name
        assert np.array_equal(order, np.argsort(-cnt, kind="stable")), name
        assert sorted(order.tolist()) == list(range(len(cnt))), name


def test_port_attention_matches_golden(golden_attention):
    for name, c in golden_attention.items():
        n, h, d = (int(x) for x in c["N"])
        o = oracle.block_attention(n, c["Q"].astype(np.float32), c["K"].astype(np.float32),
                                   c["V"].astype(np.float32), c["offsets"], c["cols"])
        # same statements, same order of float operations: bit-identical
        assert np.array_equal(o, c["O"]), (name, oracle.max_abs(o, c["O"]))


def test_port_attention_threads_identical(golden_attention):
    c = golden_attention["pl300_h1_d64"]
    args = (300, c["Q"].astype(np.float32), c["K"].astype(np.float32), c["V"].astype(np.float32),
            c["offsets"], c["cols"])
    assert np.array_equal(oracle.block_attention(*args, threads=1), oracle.block_attention(*args, threads=4))


def test_port_window_and_head_subsets(golden_attention):
    c = golden_attention["dups_unsorted_h4_d64"]
    n = int(c["N"][0])
    q, k, v = (c[x].astype(np.float32) for x in "QKV")
    full = oracle.block_attention(n, q, k, v, c["offsets"], c["cols"])
    part = oracle.block_attention(n, q, k, v, c["offsets"], c["cols"], windows=[1], heads=[2, 0])
    assert np.array_equal(part[16:32, [0, 2]], full[16:32, [0, 2]])
    assert not part[:16].any() and not part[:, 1].any()


def _random_csr(rng, n, m, shuffle=True, dups=True):
    s = rng.integers(0, n, m)
    d = rng.integers(0, n, m)
    order = np.argsort(s, kind="stable")
    s, d = s[order], d[order]
    rp = np.zeros(n + 1, np.int64)
    np.cumsum(np.bincount(s, minlength=n), out=rp[1:])
    if not dups:
        g = G.csr_from_edges(n, s, d)
        return g.row_ptr, g.col_ind
    if shuffle:
        d = d.copy()
        for u in range(n):
            seg = d[rp[u]:rp[u + 1]]
            rng.shuffle(seg)
    return rp.astype(np.int32), d.astype(np.int32)


@needs_ref
@pytest.mark.parametrize("seed", range(6))
def test_port_vs_compiled_reference_random(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 700))
    m = int(rng.integers(0, 6 * n + 1))
    rp, ci = _random_csr(rng, n, m)
    off_p, cols_p = oracle.convert(n, rp, ci)
    off_r, cols_r = oracle.ref_convert(n, rp, ci)
    assert np.array_equal(off_p, off_r) and np.array_equal(cols_p, cols_r)
    cnt = np.diff(off_r)
    assert np.array_equal(cnt[oracle.window_order(off_p)], cnt[oracle.ref_window_order(off_r)])
    d = 64
    q, k, v = (rng.uniform(-1, 1, (n, d)).astype(np.float16).astype(np.float32) for _ in range(3))
    o_p = oracle.block_attention(n, q, k, v, off_p, cols_p)[:, 0]
    o_r = oracle.ref_block_attention(n, q, k, v, off_r, cols_r)
    assert np.array_equal(o_p, o_r)
    assert np.array_equal(oracle.edge_attention(n, q, k, v, rp, ci), oracle.ref_edge_attention(n, q, k, v, rp, ci))


@needs_ref
@pytest.mark.parametrize("name", ["cora", "citeseer"])
def test_reference_datasets_digest(name):
    """The vendored Cora / Citeseer CSR (read in place from the reference
    tree) converts to the committed digests, through both the compiled
    reference and the restatement."""
    from fused3s_b200.api import load_csr_graph
    path = oracle.REFERENCE_ROOT / "data" / name
    if not path.exists():
        pytest.skip("reference data not present")
    want = json.loads((GOLDEN / "datasets.json").read_text())[name]
    g = load_csr_graph(str(path))

    def dg(*a):
        m = hashlib.sha256()
        for x in a:
            m.update(np.ascontiguousarray(x, np.int32).tobytes())
        return m.hexdigest()

    off, cols = oracle.convert(g.num_nodes, g.row_ptr, g.col_ind)
    assert dg(off, cols) == want["format_sha256"]
    assert int(cols.shape[0]) == want["num_blocks"]
    order = oracle.window_order(off)
    assert dg(np.diff(off)[order]) == want["ref_order_counts_sha256"]
    off_r, cols_r = oracle.ref_convert(g.num_nodes, g.row_ptr, g.col_ind)
    assert dg(off_r, cols_r) == want["format_sha256"]
    assert dg(oracle.ref_window_order(off_r)) == want["ref_order_sha256"]


def test_reference_loader_bug_is_fixed():
    """The reference opens col_ind.txt while its exporter writes col_idx.txt
    (include/utils.cuh:36 vs data/data_loader.py:21); our loader reads the
    file that exists."""
    from fused3s_b200.api import load_csr_graph
    path = oracle.REFERENCE_ROOT / "data" / "cora"
    if not path.exists():
        pytest.skip("reference data not present")
    g = load_csr_graph(str(path))
    assert np.count_nonzero(g.col_ind) > 0.9 * g.num_edges


def test_threaded_converter_equals_the_port():
    g = G.rmat_graph(14, 16, device="cpu", name="small-rmat")
    a = oracle.convert(g.num_nodes, g.row_ptr, g.col_ind)
    for t in (2, 7, 64):
        b = oracle.convert(g.num_nodes, g.row_ptr, g.col_ind, threads=t)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


@pytest.mark.parametrize("n", [16 * 97, 16 * 97 + 5])
def test_compact_windows_is_bit_identical_to_the_full_problem(n):
    """The sampled-window sub-problem used for large-graph parity (only the
    sampled windows and the K/V blocks they use) gives the same bits as the
    full problem, including the masked tail of the last block column."""
    rng = np.random.default_rng(n)
    src = rng.integers(0, n, 6000)
    dst = rng.integers(0, n, 6000)
    dst[:40] = n - 1  # the last (partial) block column is used
    src[40:60] = n - 1  # and the last window has rows
    g = G.csr_from_edges(n, src, dst)
    off, cols = oracle.convert(n, g.row_ptr, g.col_ind)
    H, d = 2, 64
    q, k, v = (x.float().numpy() for x in G.make_features(n, H, d, kind="uniform", seed=3))
    full = oracle.block_attention(n, q, k, v, off, cols)
    nrw = off.shape[0] - 1
    for wins in (np.array([3, 17, nrw - 1]), np.array([0, 5, 9, 44]), rng.choice(nrw, 20, replace=False)):
        c = oracle.compact_windows(n, off, cols, wins)
        qc, kc, vc = (oracle.gather_rows(x, r) for x, r in ((q, c["q_rows"]), (k, c["kv_rows"]), (v, c["kv_rows"])))
        oc = oracle.block_attention(c["num_nodes"], qc, kc, vc, c["offsets"], c["cols"], windows=c["windows"])
        for w, wc in zip(wins, c["windows"]):
            rows = np.arange(16 * w, min(16 * w + 16, n))
            crows = 16 * int(wc) + np.arange(rows.shape[0])
            assert np.array_equal(oc[crows], full[rows]), w


def test_exact_restatement_agrees_with_the_port():
    """oracle.block_attention_exact (float64, chunked) and the float32 port
    agree on ordinary windows, the masked tail included."""
    n = 16 * 60 + 7
    rng = np.random.default_rng(2)
    g = G.csr_from_edges(n, rng.integers(0, n, 3000), rng.integers(0, n, 3000))
    off, cols = oracle.convert(n, g.row_ptr, g.col_ind)
    q, k, v = (x.float().numpy() for x in G.make_features(n, 1, 64, kind="uniform", seed=4))
    ref = oracle.block_attention(n, q, k, v, off, cols)
    for w in (0, 17, len(off) - 2):
        rows = np.arange(16 * w, min(16 * w + 16, n))
        ex = oracle.block_attention_exact(n, q[rows, 0], k[:, 0], v[:, 0], off, cols, w, chunk=333)
        assert oracle.max_abs(ref[rows, 0], ex) < 1e-5
