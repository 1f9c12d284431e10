"""Seeded synthetic graphs and features standing in for the benchmark inputs.

The reference evaluates on Cora and Citeseer exported by PyG
(data/data_loader.py:6-26) and its harness draws Q/K/V from a seeded RNG
(tests/test_fused_3s_v2.cu:84-88).  The benchmark configurations C1-C5 used
here are synthetic graphs with the shapes and degree statistics of those
inputs (and three larger families); nothing here reads a dataset.

All graphs are returned as int32 CSR (row_ptr[N+1], col_ind[E]) with column
indices sorted within each row and no duplicate edges.

  C1  power-law symmetric graph, N=2708, 10,556 directed edges + self-loops
  C2  heavy-tailed sparse graph, N=3327, 9,104 directed edges + self-loops,
      ~1% isolated nodes
  C3  4096 disjoint Erdos-Renyi graphs of 20-500 nodes, mean degree 8,
      self-loops, block-diagonal
  C4  R-MAT(0.57, 0.19, 0.19, 0.05), N=2^20, average degree 16, symmetrised,
      node ids randomly permuted
  C5  the same R-MAT family, N=2^24, average degree 32
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional

import numpy as np

try:  # torch is only needed for the device-side generators (C4/C5)
    import torch
except ImportError:  # pragma: no cover
    torch = None


@dataclasses.dataclass
class CSRGraph:
    num_nodes: int
    row_ptr: np.ndarray  # int32 [N+1]
    col_ind: np.ndarray  # int32 [E]
    name: str = ""

    @property
    def num_edges(self) -> int:
        return int(self.col_ind.shape[0])


@dataclasses.dataclass
class Config:
    name: str
    heads: int
    head_dim: int
    features: str  # "uniform" (U[-1,1]) or "normal" (N(0,1)/sqrt(d))
    description: str


CONFIGS = {
    "c1": Config("c1", 1, 64, "uniform", "power-law N=2708 E~10556+self-loops, H=1 d=64"),
    "c2": Config("c2", 1, 64, "uniform", "heavy-tailed N=3327 E~9104+self-loops, 1% isolated, H=1 d=64"),
    "c3": Config("c3", 8, 64, "normal", "4096 ER graphs (20-500 nodes, deg 8)+self-loops, H=8 d=64"),
    "c4": Config("c4", 8, 64, "normal", "R-MAT N=2^20 avg deg 16 symmetrised permuted, H=8 d=64"),
    "c5": Config("c5", 4, 128, "normal", "R-MAT N=2^24 avg deg 32 symmetrised permuted, H=4 d=128"),
    # C4's family at 2^18 nodes: K+V still exceed L2 (512 MB) while the whole
    # case holds ~2 GB on the device -- the size used for ncu captures
    "c4s": Config("c4s", 8, 64, "normal", "R-MAT N=2^18 avg deg 16 symmetrised permuted, H=8 d=64"),
    # C5's family at 2^20 and 2^22 nodes (K+V 2.1 GB and 8.6 GB): the cases
    # whose DRAM traffic per block stands in for C5's in ncu captures
    "c5s": Config("c5s", 4, 128, "normal", "R-MAT N=2^20 avg deg 32 symmetrised permuted, H=4 d=128"),
    "c5m": Config("c5m", 4, 128, "normal", "R-MAT N=2^22 avg deg 32 symmetrised permuted, H=4 d=128"),
}


# ----------------------------------------------------------------------------
# CSR assembly
# ----------------------------------------------------------------------------

def csr_from_edges(num_nodes: int, src: np.ndarray, dst: np.ndarray, name: str = "") -> CSRGraph:
    """Sorted, de-duplicated int32 CSR from an edge list."""
    key = src.astype(np.int64) * num_nodes + dst.astype(np.int64)
    key = np.unique(key)
    rows = (key // num_nodes).astype(np.int64)
    cols = (key % num_nodes).astype(np.int32)
    counts = np.bincount(rows, minlength=num_nodes)
    row_ptr = np.zeros(num_nodes + 1, dtype=np.int64)
    np.cumsum(counts, out=row_ptr[1:])
    assert row_ptr[-1] < 2**31
    return CSRGraph(num_nodes, row_ptr.astype(np.int32), cols, name)


def _symmetrise(u: np.ndarray, v: np.ndarray):
    return np.concatenate([u, v]), np.concatenate([v, u])


def _with_self_loops(n: int, u: np.ndarray, v: np.ndarray):
    ids = np.arange(n, dtype=np.int64)
    return np.concatenate([u, ids]), np.concatenate([v, ids])


def _sample_weighted_pairs(rng, weights: np.ndarray, n_pairs: int, allowed: Optional[np.ndarray] = None):
    """Chung-Lu style: draw unique undirected pairs with P(u) ~ weights[u]."""
    n = weights.shape[0]
    p = weights / weights.sum()
    have = np.zeros(0, dtype=np.int64)
    while have.shape[0] < n_pairs:
        need = n_pairs - have.shape[0]
        u = rng.choice(n, size=2 * need + 64, p=p)
        v = rng.choice(n, size=2 * need + 64, p=p)
        ok = u != v
        a, b = np.minimum(u[ok], v[ok]), np.maximum(u[ok], v[ok])
        key = a.astype(np.int64) * n + b
        # keep first occurrences in draw order so the result is seed-stable
        merged = np.concatenate([have, key])
        _, first = np.unique(merged, return_index=True)
        have = merged[np.sort(first)]
    have = have[:n_pairs]
    return (have // n).astype(np.int64), (have % n).astype(np.int64)


def _capped_powerlaw_degrees(rng, n: int, exponent: float, kmin: int, kmax: int) -> np.ndarray:
    k = np.arange(kmin, kmax + 1, dtype=np.float64)
    pk = k ** (-exponent)
    pk /= pk.sum()
    return rng.choice(k, size=n, p=pk)


# ----------------------------------------------------------------------------
# C1 / C2 / C3 (host, numpy)
# ----------------------------------------------------------------------------

def powerlaw_graph(num_nodes: int = 2708, directed_edges: int = 10556, exponent: float = 2.2,
                   max_degree: int = 168, self_loops: bool = True, seed: int = 1) -> CSRGraph:
    """C1: symmetric Chung-Lu graph with a capped Zipf(exponent) weight sequence."""
    rng = np.random.default_rng(seed)
    w = _capped_powerlaw_degrees(rng, num_nodes, exponent, 1, max_degree)
    w[rng.integers(num_nodes)] = max_degree  # one hub at the cap, like Cora's max degree
    u, v = _sample_weighted_pairs(rng, w, directed_edges // 2)
    u, v = _symmetrise(u, v)
    if self_loops:
        u, v = _with_self_loops(num_nodes, u, v)
    return csr_from_edges(num_nodes, u, v, "c1")


def heavy_tailed_graph(num_nodes: int = 3327, directed_edges: int = 9104, exponent: float = 2.5,
                       max_degree: int = 99, isolated_fraction: float = 0.0144,
                       self_loops: bool = True, seed: int = 2) -> CSRGraph:
    """C2: heavy-tailed sparse graph in which ~1% of nodes have no neighbour."""
    rng = np.random.default_rng(seed)
    w = _capped_powerlaw_degrees(rng, num_nodes, exponent, 1, max_degree)
    iso = rng.choice(num_nodes, size=int(round(isolated_fraction * num_nodes)), replace=False)
    w[iso] = 0.0
    u, v = _sample_weighted_pairs(rng, w, directed_edges // 2)
    u, v = _symmetrise(u, v)
    if self_loops:
        u, v = _with_self_loops(num_nodes, u, v)
    return csr_from_edges(num_nodes, u, v, "c2")


def batched_er_graph(num_graphs: int = 4096, min_nodes: int = 20, max_nodes: int = 500,
                     mean_degree: float = 8.0, self_loops: bool = True, seed: int = 3) -> CSRGraph:
    """C3: disjoint G(n, p) graphs with p = mean_degree / (n - 1), block-diagonal."""
    rng = np.random.default_rng(seed)
    sizes = rng.integers(min_nodes, max_nodes + 1, size=num_graphs)
    base = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
    us, vs = [], []
    tri_cache = {}
    for g in range(num_graphs):
        n = int(sizes[g])
        pairs = n * (n - 1) // 2
        p = min(1.0, mean_degree / (n - 1))
        m = rng.binomial(pairs, p)
        if m == 0:
            continue
        idx = rng.choice(pairs, size=m, replace=False)
        if n not in tri_cache:
            tri_cache[n] = np.triu_indices(n, 1)
        a, b = tri_cache[n]
        us.append(a[idx] + base[g])
        vs.append(b[idx] + base[g])
    n_total = int(sizes.sum())
    u = np.concatenate(us).astype(np.int64)
    v = np.concatenate(vs).astype(np.int64)
    u, v = _symmetrise(u, v)
    if self_loops:
        u, v = _with_self_loops(n_total, u, v)
    return csr_from_edges(n_total, u, v, "c3")


def batched_er_graph_device(num_graphs: int = 4096, min_nodes: int = 20, max_nodes: int = 500,
                            mean_degree: float = 8.0, self_loops: bool = True, seed: int = 3,
                            device: str = "cuda", name: str = "c3") -> CSRGraph:
    """C3 drawn on the device: the same family as batched_er_graph (sizes
    uniform in [min_nodes, max_nodes], G(n, p) with p = mean_degree / (n - 1)
    per graph, symmetrised, self-loops, block-diagonal), vectorised over all
    graphs instead of a host loop per graph.  Every candidate pair (i < j) of
    every graph is kept with its graph's p (so each graph's edge count is
    Binomial(n (n - 1) / 2, p), as in the host version); a flat pair index is
    mapped back to (graph, i, j) with a search over the graphs' pair offsets
    and the inverse of the triangular numbering.  Deterministic for a seed
    and device type; a different draw from batched_er_graph's."""
    if torch is None:
        raise RuntimeError("batched_er_graph_device needs torch")
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    sizes = torch.randint(min_nodes, max_nodes + 1, (num_graphs,), generator=gen, device=dev, dtype=torch.int64)
    base = torch.cumsum(sizes, 0) - sizes                      # first node of each graph
    pairs = sizes * (sizes - 1) // 2
    poff = torch.cumsum(pairs, 0) - pairs                      # first flat pair of each graph
    total = int(pairs.sum())
    p = (mean_degree / (sizes - 1).clamp(min=1).to(torch.float64)).clamp(max=1.0)
    us, vs = [], []
    chunk = 1 << 26
    for s0 in range(0, total, chunk):
        idx = torch.arange(s0, min(total, s0 + chunk), device=dev, dtype=torch.int64)
        gi = torch.searchsorted(poff, idx, right=True) - 1     # graph of each pair
        keep = torch.rand(idx.shape[0], generator=gen, device=dev, dtype=torch.float64) < p[gi]
        idx, gi = idx[keep], gi[keep]
        t = idx - poff[gi]                                     # pair number inside the graph
        n = sizes[gi]
        # row i of pair t in the strict upper triangle, rows of lengths n-1, n-2, ...
        b = (2 * n - 1).to(torch.float64)
        i = torch.floor((b - torch.sqrt(b * b - 8.0 * t.to(torch.float64))) / 2).to(torch.int64)
        first = i * (2 * n - i - 1) // 2                       # first pair of row i
        i = torch.where(first > t, i - 1, i)                   # guard the float estimate
        first = i * (2 * n - i - 1) // 2
        nxt = (i + 1) * (2 * n - i - 2) // 2
        i = torch.where(t >= nxt, i + 1, i)
        first = i * (2 * n - i - 1) // 2
        j = t - first + i + 1
        us.append(base[gi] + i)
        vs.append(base[gi] + j)
    n_total = int(sizes.sum())
    u = torch.cat(us) if us else torch.zeros(0, dtype=torch.int64, device=dev)
    v = torch.cat(vs) if vs else torch.zeros(0, dtype=torch.int64, device=dev)
    src, dst = torch.cat([u, v]), torch.cat([v, u])
    if self_loops:
        ids = torch.arange(n_total, device=dev, dtype=torch.int64)
        src, dst = torch.cat([src, ids]), torch.cat([dst, ids])
    key = torch.unique(src * n_total + dst, sorted=True)
    rows = torch.div(key, n_total, rounding_mode="floor")
    cols = (key - rows * n_total).to(torch.int32)
    counts = torch.bincount(rows, minlength=n_total)
    row_ptr = torch.zeros(n_total + 1, dtype=torch.int64, device=dev)
    torch.cumsum(counts, 0, out=row_ptr[1:])
    return CSRGraph(n_total, row_ptr.to(torch.int32).cpu().numpy(), cols.cpu().numpy(), name)


# ----------------------------------------------------------------------------
# C4 / C5 (R-MAT, torch on the given device)
# ----------------------------------------------------------------------------

def rmat_graph(scale: int, avg_degree: int, a: float = 0.57, b: float = 0.19, c: float = 0.19,
               permute: bool = True, seed: int = 4, device: str = "cpu", name: str = "rmat",
               chunk: int = 1 << 26) -> CSRGraph:
    """R-MAT edges (N = 2^scale, N*avg_degree/2 draws), symmetrised, de-duplicated,
    self-loops dropped, node ids randomly permuted.  Generated with torch on
    `device` (deterministic for a given seed and device type)."""
    if torch is None:
        raise RuntimeError("rmat_graph needs torch")
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    n = 1 << scale
    m = n * avg_degree // 2
    keys = []
    perm = torch.randperm(n, generator=gen, device=dev) if permute else None
    for s in range(0, m, chunk):
        cnt = min(chunk, m - s)
        u = torch.zeros(cnt, dtype=torch.int64, device=dev)
        v = torch.zeros(cnt, dtype=torch.int64, device=dev)
        for _ in range(scale):
            r = torch.rand(cnt, generator=gen, device=dev)
            bu = (r >= a + b).to(torch.int64)
            bv = ((r >= a) & (r < a + b)) | (r >= a + b + c)
            u = u * 2 + bu
            v = v * 2 + bv.to(torch.int64)
        if perm is not None:
            u = perm[u]
            v = perm[v]
        keep = u != v
        u, v = u[keep], v[keep]
        keys.append(torch.cat([u * n + v, v * n + u]))
        del u, v, keep
    key = torch.unique(torch.cat(keys), sorted=True)
    del keys
    rows = torch.div(key, n, rounding_mode="floor")
    cols = (key - rows * n).to(torch.int32)
    counts = torch.bincount(rows, minlength=n)
    row_ptr = torch.zeros(n + 1, dtype=torch.int64, device=dev)
    torch.cumsum(counts, 0, out=row_ptr[1:])
    assert int(row_ptr[-1]) < 2**31
    return CSRGraph(n, row_ptr.to(torch.int32).cpu().numpy(), cols.cpu().numpy(), name)


def make_graph(config: str, device: str = "cpu", seed: Optional[int] = None) -> CSRGraph:
    """The graph of one benchmark configuration (c1..c5)."""
    kw = {} if seed is None else {"seed": seed}
    if config == "c1":
        return powerlaw_graph(**kw)
    if config == "c2":
        return heavy_tailed_graph(**kw)
    if config == "c3":
        if device != "cpu":  # drawn on the GPU (the host loop stays for CPU callers)
            return batched_er_graph_device(device=device, **kw)
        return batched_er_graph(**kw)
    if config == "c4":
        return rmat_graph(20, 16, device=device, name="c4", **kw)
    if config == "c5":
        return rmat_graph(24, 32, device=device, name="c5", **kw)
    if config == "c4s":
        return rmat_graph(18, 16, device=device, name="c4s", **kw)
    if config == "c5s":
        return rmat_graph(20, 32, device=device, name="c5s", **kw)
    if config == "c5m":
        return rmat_graph(22, 32, device=device, name="c5m", **kw)
    raise ValueError(f"unknown config {config!r}")


# ----------------------------------------------------------------------------
# Features
# ----------------------------------------------------------------------------

def make_features(num_nodes: int, heads: int, head_dim: int, kind: str = "uniform",
                  seed: int = 42, device: str = "cpu"):
    """Q, K, V as fp16 torch tensors of shape [num_nodes, heads, head_dim].

    kind "uniform": fp32 U[-1, 1] cast to fp16 (C1, C2).
    kind "normal":  fp32 N(0, 1) / sqrt(head_dim) cast to fp16 (C3-C5).
    """
    if torch is None:
        raise RuntimeError("make_features needs torch")
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    shape = (num_nodes, heads, head_dim)
    out = []
    for _ in range(3):
        if kind == "uniform":
            x = torch.rand(shape, generator=gen, device=dev, dtype=torch.float32) * 2.0 - 1.0
        elif kind == "normal":
            x = torch.randn(shape, generator=gen, device=dev, dtype=torch.float32) / math.sqrt(head_dim)
        else:
            raise ValueError(kind)
        out.append(x.to(torch.float16))
    return tuple(out)


def make_features_device(num_nodes: int, heads: int, head_dim: int, kind: str = "normal", seed: int = 42,
                         device="cuda"):
    """fp16 [num_nodes, heads, head_dim] Q, K, V drawn on the device in row
    chunks (no fp32 copy of a whole tensor), for the large configurations.
    Same distributions as make_features; the values depend on the chunking,
    so they differ from make_features' for the same seed."""
    if torch is None:
        raise RuntimeError("make_features_device needs torch")
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    out = []
    chunk = max(1, (1 << 27) // (heads * head_dim))
    for _ in range(3):
        t = torch.empty((num_nodes, heads, head_dim), dtype=torch.float16, device=dev)
        for r in range(0, num_nodes, chunk):
            rr = min(num_nodes, r + chunk)
            if kind == "uniform":
                x = torch.rand((rr - r, heads, head_dim), generator=gen, device=dev) * 2 - 1
            elif kind == "normal":
                x = torch.randn((rr - r, heads, head_dim), generator=gen, device=dev) / math.sqrt(head_dim)
            else:
                raise ValueError(kind)
            t[r:rr] = x.to(torch.float16)
        out.append(t)
    return tuple(out)


def graph_stats(g: CSRGraph) -> dict:
    deg = np.diff(g.row_ptr.astype(np.int64))
    return {
        "num_nodes": g.num_nodes,
        "num_edges": g.num_edges,
        "max_degree": int(deg.max()) if deg.size else 0,
        "mean_degree": float(deg.mean()) if deg.size else 0.0,
        "zero_degree": int((deg == 0).sum()),
    }
