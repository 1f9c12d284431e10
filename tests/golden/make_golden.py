"""Generate the golden fixtures in tests/golden/ from the REFERENCE's own code.

    make -C oracle all        # builds oracle/_ref/libf3s_ref.so from the reference sources
    python tests/golden/make_golden.py

Every expected output here comes from the reference functions compiled
unchanged (oracle/_ref): convert_csr_to_block_sparse (src/converter.cu:13),
generate_balanced_window_order (include/utils.cuh:48, libstdc++ std::sort)
and cpu_block_sparse_attention (tests/test_fused_3s_v2.cu:17).  Inputs are
seeded synthetic graphs and fp16-representable features (stored in the
fixture, so the files do not depend on any RNG implementation).

Fixtures:
  graphs.npz     per case: N, row_ptr, col_ind, offsets, cols, ref_order
  attention.npz  per case: N, H, d, Q, K, V (fp16), O (fp32, per head from
                 the reference function), and the case's format
  datasets.json  digests of the reference converter output and order on the
                 reference's vendored Cora / Citeseer CSR (read in place)
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from fused3s_b200 import graphs as G  # noqa: E402

OUT = Path(__file__).resolve().parent


def edge_case_graphs():
    """Small graphs covering the converter's edge cases."""
    rng = np.random.default_rng(7)
    cases = {}

    def add(name, n, src, dst, sort_rows=True, dedupe=True):
        src = np.asarray(src, np.int64)
        dst = np.asarray(dst, np.int64)
        if dedupe:
            g = G.csr_from_edges(n, src, dst)
            rp, ci = g.row_ptr, g.col_ind
        else:  # keep duplicates / original order inside rows
            order = np.argsort(src, kind="stable")
            src, dst = src[order], dst[order]
            counts = np.bincount(src, minlength=n)
            rp = np.zeros(n + 1, np.int64)
            np.cumsum(counts, out=rp[1:])
            rp, ci = rp.astype(np.int32), dst.astype(np.int32)
        if not sort_rows:  # shuffle columns inside each row
            ci = ci.copy()
            for u in range(n):
                seg = ci[rp[u]:rp[u + 1]]
                rng.shuffle(seg)
        cases[name] = (n, rp.astype(np.int32), ci.astype(np.int32))

    add("single_node", 1, [0], [0])
    add("n15_dense", 15, *np.nonzero(np.ones((15, 15))))
    add("n16_ring", 16, np.arange(16), (np.arange(16) + 1) % 16)
    add("n17_star", 17, np.r_[np.zeros(16), np.arange(1, 17)], np.r_[np.arange(1, 17), np.zeros(16)])
    # empty windows: only nodes 0..15 and 48..63 have edges (windows 1, 2 and 4 empty)
    s = np.r_[rng.integers(0, 16, 40), rng.integers(48, 64, 40)]
    add("empty_windows", 80, s, rng.integers(0, 80, 80))
    # duplicate edges and unsorted rows, 33 nodes (tail of 1 row)
    s = rng.integers(0, 33, 300)
    add("dups_unsorted", 33, s, rng.integers(0, 33, 300), sort_rows=False, dedupe=False)
    # isolated nodes with self-loops only, N % 16 == 12
    n = 300
    s = rng.integers(0, n, 900)
    d = rng.integers(0, n, 900)
    keep = (s % 7) != 0  # nodes divisible by 7 keep only their self-loop
    s, d = s[keep], d[keep]
    s, d = np.r_[s, d, np.arange(n)], np.r_[d, s, np.arange(n)]
    add("isolated_selfloops", n, s, d)
    # one heavy window (> 4096 edges) next to light ones
    n = 9000
    hub = np.repeat(np.arange(16), 400)
    s = np.r_[hub, rng.integers(16, n, 3000)]
    d = np.r_[rng.permutation(n)[:6400] % n, rng.integers(0, n, 3000)]
    add("heavy_window", n, s, d, dedupe=False)
    return cases


def attention_cases():
    """(name, N, H, d, graph) for the attention fixtures."""
    g300 = G.powerlaw_graph(num_nodes=300, directed_edges=1400, max_degree=60, seed=11)
    g200 = G.heavy_tailed_graph(num_nodes=200, directed_edges=700, max_degree=40, seed=12)
    g150 = G.powerlaw_graph(num_nodes=150, directed_edges=600, max_degree=40, seed=13)
    g_empty = edge_case_graphs()["empty_windows"]
    g_dups = edge_case_graphs()["dups_unsorted"]
    return [
        ("pl300_h1_d64", 300, 1, 64, (g300.num_nodes, g300.row_ptr, g300.col_ind)),
        ("ht200_h2_d64", 200, 2, 64, (g200.num_nodes, g200.row_ptr, g200.col_ind)),
        ("pl150_h1_d128", 150, 1, 128, (g150.num_nodes, g150.row_ptr, g150.col_ind)),
        ("empty_windows_h1_d64", 80, 1, 64, g_empty),
        ("dups_unsorted_h4_d64", 33, 4, 64, g_dups),
    ]


def features(n, h, d, seed):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(3):
        x = rng.uniform(-1.0, 1.0, size=(n, h, d)).astype(np.float16)
        out.append(x)
    return out


def digest(*arrays) -> str:
    m = hashlib.sha256()
    for a in arrays:
        m.update(np.ascontiguousarray(a, np.int32).tobytes())
    return m.hexdigest()


def main():
    if not oracle.ref_available():
        raise SystemExit("build oracle/_ref first: make -C oracle all")
    graphs = {}
    cases = edge_case_graphs()
    cases["c1"] = (lambda g: (g.num_nodes, g.row_ptr, g.col_ind))(G.make_graph("c1"))
    cases["c2"] = (lambda g: (g.num_nodes, g.row_ptr, g.col_ind))(G.make_graph("c2"))
    for name, (n, rp, ci) in cases.items():
        off, cols = oracle.ref_convert(n, rp, ci)
        order = oracle.ref_window_order(off)
        graphs[f"{name}/N"] = np.array([n], np.int64)
        graphs[f"{name}/row_ptr"] = rp
        graphs[f"{name}/col_ind"] = ci
        graphs[f"{name}/offsets"] = off
        graphs[f"{name}/cols"] = cols
        graphs[f"{name}/ref_order"] = order
    np.savez_compressed(OUT / "graphs.npz", **graphs)

    att = {}
    for i, (name, n, h, d, (gn, rp, ci)) in enumerate(attention_cases()):
        assert gn == n
        off, cols = oracle.ref_convert(n, rp, ci)
        q, k, v = features(n, h, d, seed=100 + i)
        o = np.zeros((n, h, d), np.float32)
        for hh in range(h):
            o[:, hh, :] = oracle.ref_block_attention(
                n, q[:, hh, :].astype(np.float32), k[:, hh, :].astype(np.float32),
                v[:, hh, :].astype(np.float32), off, cols)
        for key, val in (("N", np.array([n, h, d], np.int64)), ("row_ptr", rp), ("col_ind", ci),
                         ("offsets", off), ("cols", cols), ("Q", q), ("K", k), ("V", v), ("O", o)):
            att[f"{name}/{key}"] = val
    np.savez_compressed(OUT / "attention.npz", **att)

    ds = {}
    from fused3s_b200.api import load_csr_graph
    for name in ("cora", "citeseer"):
        path = oracle.REFERENCE_ROOT / "data" / name
        if not path.exists():
            continue
        g = load_csr_graph(str(path))
        off, cols = oracle.ref_convert(g.num_nodes, g.row_ptr, g.col_ind)
        order = oracle.ref_window_order(off)
        ds[name] = {
            "num_nodes": g.num_nodes,
            "num_edges": g.num_edges,
            "num_blocks": int(cols.shape[0]),
            "format_sha256": digest(off, cols),
            "ref_order_sha256": digest(order),
            "ref_order_counts_sha256": digest(np.diff(off)[order]),
        }
    (OUT / "datasets.json").write_text(json.dumps(ds, indent=1) + "\n")
    for p in ("graphs.npz", "attention.npz", "datasets.json"):
        print(p, (OUT / p).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
