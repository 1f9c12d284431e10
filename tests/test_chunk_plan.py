"""Column-chunked work plans built on the host (column_chunk_pieces):
against a direct loop, and the invariants the kernels rely on (pieces
cover every listed window's blocks once, stay inside one column chunk and
one window, come chunk by chunk; a split window's pieces own consecutive
slots in column order)."""
import numpy as np
import pytest

import oracle
from fused3s_b200.api import column_chunk_pieces
from fused3s_b200 import graphs as G


def _loop(off, cols, order, cw, T):
    items = []  # per listed index: list of (chunk, lo, hi)
    for w in order:
        b0, b1 = off[w], off[w + 1]
        ps = []
        b = b0
        while b < b1:
            c = cols[b] // cw
            e = b
            while e < b1 and cols[e] // cw == c:
                e += 1
            for s in range(b, e, T if T else e - b):
                ps.append((c, s, min(e, s + T) if T else e))
            b = e
        items.append(ps)
    pieces, splits, slot = [], [], 0
    slots = []
    for i, (w, ps) in enumerate(zip(order, items)):
        if len(ps) > 1:
            splits.append((w, slot, len(ps), 0))
            slots.append(list(range(slot, slot + len(ps))))
            slot += len(ps)
        else:
            slots.append([-1] * len(ps))
    chunks = sorted({c for ps in items for c, _, _ in ps} | {0})
    for c in chunks:
        for i, (w, ps) in enumerate(zip(order, items)):
            for k, (cc, lo, hi) in enumerate(ps):
                if cc == c:
                    pieces.append((w, lo, hi, slots[i][k]))
        if c == 0:  # windows without blocks: one empty piece each, with chunk 0
            for w, ps in zip(order, items):
                if not ps:
                    pieces.append((w, off[w], off[w], -1))
    return np.array(pieces, np.int32).reshape(-1, 4), np.array(splits, np.int32).reshape(-1, 4), slot


@pytest.mark.parametrize("cw,T", [(1, 0), (4, 0), (8, 3), (1000, 0), (3, 1)])
def test_chunk_pieces_match_loop(cw, T):
    g = G.powerlaw_graph(num_nodes=1203, directed_edges=9000, max_degree=300, seed=cw + T)
    off, cols = oracle.convert(g.num_nodes, g.row_ptr, g.col_ind)
    order = oracle.window_order(off)
    got = column_chunk_pieces(off, cols, order, cw, T)
    want = _loop(off, cols, order, cw, T)
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1]) and got[2] == want[2]


def test_chunk_pieces_invariants_with_empty_windows_and_subsets():
    rng = np.random.default_rng(3)
    n = 16 * 300
    src = rng.integers(0, n, 20000)
    src[src // 16 % 7 == 0] = 5  # many windows without blocks
    g = G.csr_from_edges(n, src, rng.integers(0, n, 20000))
    off, cols = oracle.convert(n, g.row_ptr, g.col_ind)
    order = oracle.window_order(off)[::2]  # a subset of the windows
    pieces, splits, n_slots, starts = column_chunk_pieces(off, cols, order, 16, 5)
    cw = 16
    # the chunk ranges partition the pieces, each range one column chunk
    assert starts[0] == 0 and starts[-1] == pieces.shape[0]
    for c in range(starts.shape[0] - 1):
        for w, lo, hi, s in pieces[starts[c]:starts[c + 1]]:
            if hi > lo:
                assert cols[lo] // cw == c
    covered = {}
    for w, lo, hi, s in pieces:
        assert off[w] <= lo <= hi <= off[w + 1]
        if hi > lo:
            assert cols[lo] // cw == cols[hi - 1] // cw and hi - lo <= 5
        covered.setdefault(w, []).append((lo, hi))
    assert set(covered) == set(order.tolist())
    for w, rngs in covered.items():
        blocks = sorted(b for lo, hi in rngs for b in range(lo, hi))
        assert blocks == list(range(off[w], off[w + 1]))
    chunk_seq = [cols[lo] // cw for w, lo, hi, s in pieces if hi > lo]
    assert chunk_seq == sorted(chunk_seq)
    used = sorted(s for *_, s in pieces if s >= 0)
    assert used == list(range(n_slots))
    for w, first, cnt, _ in splits:
        mine = sorted((lo, s) for ww, lo, hi, s in pieces if ww == w)
        assert [s for _, s in mine] == list(range(first, first + cnt))


def test_explicit_cuts_equal_multiples_and_cover_uneven_slices():
    g = G.powerlaw_graph(num_nodes=1203, directed_edges=9000, max_degree=300, seed=11)
    off, cols = oracle.convert(g.num_nodes, g.row_ptr, g.col_ind)
    order = oracle.window_order(off)
    nrw = off.shape[0] - 1
    a = column_chunk_pieces(off, cols, order, 8, 0)
    b = column_chunk_pieces(off, cols, order, col_cuts=np.arange(0, nrw + 8, 8))
    for x, y in zip(a[:2], b[:2]):
        assert np.array_equal(x, y)
    assert a[2] == b[2]
    # uneven slices (the K / V slices of a ring of 3 GPUs)
    cuts = np.array([0, nrw // 3, (2 * nrw) // 3, nrw])
    pieces, splits, n_slots, starts = column_chunk_pieces(off, cols, order, col_cuts=cuts)
    for j in range(3):
        for w, lo, hi, s in pieces[starts[j]:starts[j + 1]]:
            if hi > lo:
                assert cuts[j] <= cols[lo] and cols[hi - 1] < cuts[j + 1]
    blocks = sorted(b for w, lo, hi, s in pieces for b in range(lo, hi))
    assert blocks == list(range(off[-1]))
    with pytest.raises(ValueError):
        column_chunk_pieces(off, cols, order, col_cuts=np.array([0, nrw // 2]))  # does not cover


def test_locality_order_is_a_permutation_heavy_first():
    """api.locality_order on CPU tensors: a permutation of the listed
    windows; windows above the threshold first, heaviest first with ties in
    their listed order; then every other window in ascending id."""
    import types

    import torch

    from fused3s_b200 import api

    rng = np.random.default_rng(3)
    cnt = rng.integers(0, 40, 500)
    cnt[[7, 90, 91, 300]] = 200  # ties among heavy windows
    off = torch.from_numpy(np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32))
    fmt = types.SimpleNamespace(window_offsets=off, num_row_windows=500)
    for subset in (None, torch.from_numpy(rng.permutation(500)[:300].astype(np.int32))):
        got = api.locality_order(fmt, 30, order=subset).numpy()
        wins = np.arange(500) if subset is None else subset.numpy()
        assert sorted(got.tolist()) == sorted(wins.tolist())
        heavy = [w for w in wins if cnt[w] > 30]
        pos = {int(w): i for i, w in enumerate(wins)}
        want_heavy = sorted(heavy, key=lambda w: (-cnt[w], pos[int(w)]))
        want_light = sorted(w for w in wins if cnt[w] <= 30)
        assert got.tolist() == [int(w) for w in want_heavy + want_light]
