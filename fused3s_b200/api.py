"""Python host API of the B200 fused 3S engine.

It mirrors the reference's host interface for the fused3s_v2 path, with the
same names and argument meanings, computed on the GPU through the C ABI of
libfused3s.so (include/fused3s.h):

  GraphData, load_csr_graph            include/utils.cuh:19-40
  BlockSparseFormat                    include/utils.cuh:42-46 (blockSparseFormat)
  convert_csr_to_block_sparse          src/converter.cu:13-44
  generate_balanced_window_order       include/utils.cuh:48-59
  f3s_1tb1rw_kernel                    src/fused3s_v2.cu:81-90 (same argument list)
  float2half                           tests/test_fused_3s_v2.cu:61-64

plus the extended forward `fused3s_forward` (true num_nodes with masking of
columns >= N, H heads, head_dim 64/128, window subsets for sharding).

Differences from the reference, each deliberate:
  * errors raise Fused3SError instead of exit() (CUDA_CHECK, utils.cuh:9-17);
  * load_csr_graph reads col_idx.txt, the name data/data_loader.py writes
    (the reference opens col_ind.txt and silently reads zeros, utils.cuh:36);
  * the window order breaks ties by ascending window id (stable); the block
    count sequence along the order equals the reference's std::sort result.
"""
from __future__ import annotations

import dataclasses
import os
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import Fused3SError, check


# ----------------------------------------------------------------------------
# containers
# ----------------------------------------------------------------------------

@dataclasses.dataclass
class GraphData:
    """CSR graph (include/utils.cuh:19-24)."""
    num_nodes: int
    num_edges: int
    row_ptr: "np.ndarray | torch.Tensor"  # int32 [num_nodes + 1] (host, or device from load_csr_graph_device)
    col_ind: "np.ndarray | torch.Tensor"  # int32 [num_edges]


@dataclasses.dataclass
class BlockSparseFormat:
    """16x16 block-sparse row windows (include/utils.cuh:42-46), device-resident."""
    num_row_windows: int
    window_offsets: torch.Tensor     # int32 [nrw + 1] on the GPU
    block_col_indices: torch.Tensor  # int32 [B] on the GPU
    num_nodes: int
    # buffer behind block_col_indices (never empty, so its pointer is valid
    # even for a graph without edges)
    storage: Optional[torch.Tensor] = None

    @property
    def cols_ptr(self) -> int:
        buf = self.storage if self.storage is not None else self.block_col_indices
        if buf.numel() == 0:
            buf = self.storage = torch.zeros(1, dtype=torch.int32, device=buf.device)
        return buf.data_ptr()

    @property
    def num_blocks(self) -> int:
        return int(self.block_col_indices.shape[0])

    def to_host(self):
        return (self.window_offsets.cpu().numpy(), self.block_col_indices.cpu().numpy())


def load_csr_graph(dataset_dir: str) -> GraphData:
    """Read meta.txt / row_ptr.txt / col_idx.txt written by the reference's
    data/data_loader.py (include/utils.cuh:26-40, with the column file name
    fixed; col_ind.txt is accepted too)."""
    with open(os.path.join(dataset_dir, "meta.txt")) as f:
        num_nodes, num_edges = (int(x) for x in f.read().split()[:2])
    row_ptr = np.loadtxt(os.path.join(dataset_dir, "row_ptr.txt"), dtype=np.int64).reshape(-1)
    col_path = os.path.join(dataset_dir, "col_idx.txt")
    if not os.path.exists(col_path):
        col_path = os.path.join(dataset_dir, "col_ind.txt")
    col_ind = np.loadtxt(col_path, dtype=np.int64).reshape(-1)
    if row_ptr.shape[0] != num_nodes + 1 or col_ind.shape[0] != num_edges:
        raise ValueError(f"{dataset_dir}: sizes disagree with meta.txt")
    return GraphData(num_nodes, num_edges, row_ptr.astype(np.int32), col_ind.astype(np.int32))


# ----------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------

def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


class _WorkspaceCache:
    """Grow-only device workspaces, one per (device, stream, purpose)."""

    def __init__(self):
        self._ws = {}

    def get(self, device: torch.device, kind: str, nbytes: int) -> torch.Tensor:
        key = (device.index, _stream_ptr(device), kind)
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws


_WS = _WorkspaceCache()


def _as_device_i32(x, device: torch.device) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x.to(device=device, dtype=torch.int32).contiguous()
    return torch.from_numpy(np.ascontiguousarray(np.asarray(x, dtype=np.int32))).to(device)


def _default_device(device) -> torch.device:
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("fused3s_b200 runs on CUDA devices only (no CPU fallback)")
    return device


# ----------------------------------------------------------------------------
# converter / order
# ----------------------------------------------------------------------------

_TEXT_CHUNK = (1 << 31) - 2  # f3s_parse_int32 takes fewer bytes per call
_TEXT_SEPARATORS = np.frombuffer(b" \t\r\n", dtype=np.uint8)


def text_pieces(host_text: np.ndarray, limit: int = _TEXT_CHUNK):
    """[start, end) byte ranges of at most `limit` bytes that cover the text
    and end just after a separator (except the last), so no number is cut."""
    n = int(host_text.shape[0])
    cuts, start = [], 0
    while start < n:
        end = min(n, start + limit)
        if end < n:
            seps = np.flatnonzero(np.isin(host_text[start:end], _TEXT_SEPARATORS))
            if seps.size == 0:
                raise ValueError("text has a token longer than one parse call")
            end = start + int(seps[-1]) + 1
        cuts.append((start, end))
        start = end
    return cuts


def parse_int32_text(text, max_count: Optional[int] = None, device=None) -> torch.Tensor:
    """Whitespace-separated decimal integers decoded on the GPU
    (f3s_parse_int32).  `text`: bytes, a numpy uint8 array or a uint8 tensor
    (host or device).  Returns int32 values on `device`.  Texts longer than
    one call takes are cut at a separator (text_pieces) and decoded piece by
    piece."""
    lib = _lib.load()
    device = _default_device(device)
    if isinstance(text, (bytes, bytearray, memoryview)):
        text = np.frombuffer(bytes(text), dtype=np.uint8)
    if isinstance(text, np.ndarray):
        host = text.view(np.uint8).reshape(-1)
        if not host.flags.writeable:  # e.g. a view of bytes; torch wants writable memory
            host = host.copy()
        dev_text = torch.from_numpy(host).to(device)
    else:
        dev_text = text.to(device=device, dtype=torch.uint8).contiguous().view(-1)
        host = None
    n = int(dev_text.numel())
    if n > _TEXT_CHUNK and host is None:
        host = dev_text.cpu().numpy()
    pieces = text_pieces(host) if host is not None else [(0, n)] if n else []
    cap = (n + 1) // 2 if max_count is None else int(max_count)
    out = torch.empty(max(cap, 1), dtype=torch.int32, device=device)
    got = 0
    for start, end in pieces:
        nb = end - start
        ws = _WS.get(device, "text", lib.f3s_parse_int32_workspace_size(nb))
        cnt = _lib.ctypes.c_int64(0)
        with torch.cuda.device(device):
            st = lib.f3s_parse_int32(dev_text.data_ptr() + start, nb, out.data_ptr() + 4 * got, cap - got, cnt,
                                     _ptr(ws), ws.numel(), _stream_ptr(device))
        check(st, "f3s_parse_int32")
        got += cnt.value
    return out[:got]


def load_csr_graph_device(dataset_dir: str, device=None) -> GraphData:
    """load_csr_graph with the text decoded on the GPU: the files' bytes go to
    the device as they are (include/utils.cuh:26-40, column file col_idx.txt
    or col_ind.txt).  Returns GraphData whose row_ptr / col_ind are int32
    device tensors, ready for convert_csr_to_block_sparse."""
    device = _default_device(device)
    with open(os.path.join(dataset_dir, "meta.txt")) as f:
        num_nodes, num_edges = (int(x) for x in f.read().split()[:2])
    col_path = os.path.join(dataset_dir, "col_idx.txt")
    if not os.path.exists(col_path):
        col_path = os.path.join(dataset_dir, "col_ind.txt")
    row_ptr = parse_int32_text(np.fromfile(os.path.join(dataset_dir, "row_ptr.txt"), dtype=np.uint8),
                               num_nodes + 1, device)
    col_ind = parse_int32_text(np.fromfile(col_path, dtype=np.uint8), num_edges, device)
    if row_ptr.numel() != num_nodes + 1 or col_ind.numel() != num_edges:
        raise ValueError(f"{dataset_dir}: sizes disagree with meta.txt")
    return GraphData(num_nodes, num_edges, row_ptr, col_ind)


def convert_csr_to_block_sparse(num_nodes: int, row_ptr, col_ind, device=None) -> BlockSparseFormat:
    """CSR -> block-sparse row windows on the GPU (src/converter.cu:13-44).

    Bit-exact to the reference converter.  Raises Fused3SError with
    F3S_ERR_BAD_CSR on a column outside [0, N) or a decreasing row_ptr.
    Synchronises (returns exact-size arrays)."""
    lib = _lib.load()
    device = _default_device(device)
    rp = _as_device_i32(row_ptr, device)
    ci = _as_device_i32(col_ind, device)
    nnz = int(ci.numel())
    if rp.numel() != num_nodes + 1:
        raise ValueError("row_ptr must have num_nodes + 1 entries")
    nrw = (num_nodes + 15) // 16
    offsets = torch.empty(nrw + 1, dtype=torch.int32, device=device)
    cols = torch.empty(max(nnz, 1), dtype=torch.int32, device=device)
    wsz = lib.f3s_convert_workspace_size(num_nodes, nnz)
    ws = _WS.get(device, "convert", wsz)
    nb = _lib._I64(0)
    with torch.cuda.device(device):
        st = lib.f3s_convert(_ptr(rp), _ptr(ci) if nnz else None, num_nodes, nnz, _ptr(offsets),
                             _ptr(cols), _ptr(ws), ws.numel(), nb, _stream_ptr(device))
    check(st, "f3s_convert")
    return BlockSparseFormat(nrw, offsets, cols[: nb.value], num_nodes, storage=cols)


def generate_balanced_window_order(fmt: BlockSparseFormat) -> torch.Tensor:
    """Window ids sorted by active-block count, descending (include/utils.cuh:48-59)."""
    lib = _lib.load()
    device = fmt.window_offsets.device
    order = torch.empty(max(fmt.num_row_windows, 1), dtype=torch.int32, device=device)
    ws = _WS.get(device, "order", lib.f3s_window_order_workspace_size(fmt.num_row_windows))
    with torch.cuda.device(device):
        st = lib.f3s_window_order(_ptr(fmt.window_offsets), fmt.num_row_windows, _ptr(order), _ptr(ws),
                                  ws.numel(), _stream_ptr(device))
    check(st, "f3s_window_order")
    return order[: fmt.num_row_windows]


def locality_order(fmt: BlockSparseFormat, heavy_blocks: int, order: Optional[torch.Tensor] = None) -> torch.Tensor:
    """A work order for the fused forward that keeps neighbouring windows
    together: the windows with more than `heavy_blocks` blocks first, heaviest
    first (they bound the tail, as in the balanced order; equal counts keep
    their order in `order`, ascending id for the default and for the
    balanced order), then every other window in ascending id.  Neighbouring windows of a graph whose nodes are
    numbered by locality (communities, block-diagonal batches) share block
    columns, so they then run at the same time and their K / V tiles are
    reused from L2; the result is the same as for any other order (windows
    write disjoint rows).  `order` restricts it to those windows (a rank's
    share); default all windows."""
    device = fmt.window_offsets.device
    off = fmt.window_offsets
    if order is None:
        wins = torch.arange(fmt.num_row_windows, dtype=torch.int64, device=device)
    else:
        wins = order.to(device=device, dtype=torch.int64)
    cnt = (off[wins + 1] - off[wins]).to(torch.int64)
    heavy = cnt > heavy_blocks
    hw, hc = wins[heavy], cnt[heavy]
    # heaviest first; ties keep their listed order (a stable sort by -count)
    idx = torch.sort(-hc, stable=True).indices if hw.numel() else hc
    light = torch.sort(wins[~heavy]).values
    return torch.cat([hw[idx], light]).to(torch.int32).contiguous()


# ----------------------------------------------------------------------------
# fused forward
# ----------------------------------------------------------------------------

def _check_features(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor):
    for name, t in (("Q", Q), ("K", K), ("V", V)):
        if t.dtype != torch.float16:
            raise TypeError(f"{name} must be float16")
        if t.device.type != "cuda":
            raise ValueError(f"{name} must be on a CUDA device")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if K.shape != V.shape:
        raise ValueError("K and V must have the same shape")


def _as_nhd(t: torch.Tensor) -> torch.Tensor:
    return t.unsqueeze(1) if t.dim() == 2 else t


def block_hints(fmt: BlockSparseFormat, heads: int, head_dim: int, order: Optional[torch.Tensor] = None,
                l2_fraction: float = 0.5) -> torch.Tensor:
    """L2 eviction hints, one per active block (uint8[num_blocks]), for the
    windows in `order` (default: all).  A block's hint is its column's: the
    most popular block columns that fit in `l2_fraction` of the device's L2
    are kept, columns used by a single listed window streamed.  Computed once
    per graph; pass to fused3s_forward(block_hints=...)."""
    lib = _lib.load()
    device = fmt.window_offsets.device
    nrw = fmt.num_row_windows
    if order is None:
        order = torch.arange(nrw, dtype=torch.int32, device=device)
    order = order.to(device=device, dtype=torch.int32).contiguous()
    nb = int(fmt.num_blocks)
    hints = torch.zeros(max(nb, 1), dtype=torch.uint8, device=device)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    ws = _WS.get(device, "hints", lib.f3s_block_hints_workspace_size(nrw))
    with torch.cuda.device(device):
        st = lib.f3s_block_hints(_ptr(fmt.window_offsets), fmt.cols_ptr, _ptr(order), int(order.numel()), nrw,
                                 16 * heads * head_dim * 2 * 2, int(l2 * l2_fraction), _ptr(hints), _ptr(ws),
                                 ws.numel(), _stream_ptr(device))
    check(st, "f3s_block_hints")
    return hints[:nb]


@dataclasses.dataclass
class ForwardPlan:
    """Device-resident work plan (f3s_make_plan): the listed windows in
    order, heavy ones cut into pieces of at most `max_blocks` blocks.
    piece_ranges: for a plan cut at K / V slice boundaries (make_sliced_plan),
    the [begin, end) pieces of each slice.  sweep: a window's pieces run in
    sequence within one launch, carrying its running state (make_sweep_plan)."""
    buffer: torch.Tensor
    heads: int
    head_dim: int
    max_blocks: int
    piece_ranges: Optional[list] = None
    sweep: bool = False  # a sweep plan (make_sweep_plan): needs the larger workspace


# Longest run of blocks one work item accumulates.  The tensor cores add each
# block's P.V into the fp32 O accumulator with truncation (round toward
# zero), so an accumulator fed n blocks in a row drifts toward zero by about
# n * 2^-26 of its value; hub windows of hundreds of thousands of blocks
# would lose ~0.4 % (measured on C5).  Pieces of at most this many blocks are
# merged with round-to-nearest fp32 arithmetic (k_merge_pieces), which keeps
# the drift near 1e-4.
MAX_PIECE_BLOCKS = 4096


def auto_piece_blocks(num_blocks: int, device=None) -> int:
    """Piece size: a quarter of one SM's share of the blocks, so no single
    window can hold one SM much past the others, at most MAX_PIECE_BLOCKS
    (accumulation accuracy of hub windows) and never below 16 blocks (a
    piece's partial state is about one block's K/V bytes, so a piece of 16
    blocks moves at most ~6 % more)."""
    device = _default_device(device)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return max(16, min(MAX_PIECE_BLOCKS, -(-int(num_blocks) // (4 * sms))))


def make_plan(fmt: BlockSparseFormat, heads: int, head_dim: int, order: Optional[torch.Tensor] = None,
              max_blocks: Optional[int] = None) -> ForwardPlan:
    """Plan for fused3s_forward over the windows in `order` (default: the
    balanced order of all windows).  max_blocks: piece size (default
    auto_piece_blocks of the listed windows' blocks)."""
    lib = _lib.load()
    device = fmt.window_offsets.device
    if order is None:
        order = generate_balanced_window_order(fmt)
        nb = max(fmt.num_blocks, 1)
    else:
        order = order.to(device=device, dtype=torch.int32).contiguous()
        off = fmt.window_offsets
        nb = max(int((off[order.long() + 1] - off[order.long()]).sum().item()) if order.numel() else 0, 1)
    order = order.to(device=device, dtype=torch.int32).contiguous()
    n = int(order.numel())
    if max_blocks is None:
        max_blocks = auto_piece_blocks(nb, device)
    size = lib.f3s_plan_size(n, nb, int(max_blocks), heads, head_dim)
    if size == 0:
        raise ValueError("unsupported plan parameters")
    buf = torch.empty(size, dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        st = lib.f3s_make_plan(_ptr(fmt.window_offsets), _ptr(order), n, nb, int(max_blocks), heads, head_dim,
                               _ptr(buf), size, _stream_ptr(device))
    check(st, "f3s_make_plan")
    return ForwardPlan(buf, heads, head_dim, int(max_blocks))


def column_chunk_pieces(window_offsets: np.ndarray, block_cols: np.ndarray, order: np.ndarray, chunk_cols: int = 0,
                        max_blocks: int = 0, col_cuts=None):
    """Pieces of a column-chunked plan, built on the host.

    Every listed window's blocks (sorted by column) are cut where the block
    column crosses a chunk boundary -- a multiple of `chunk_cols`, or the
    explicit ascending boundaries `col_cuts` (first 0, last >= the number of
    block columns) -- and runs longer than `max_blocks` (0: no limit) every
    `max_blocks` blocks.  Pieces are ordered chunk by chunk, windows in
    `order` within a chunk, so all SMs read one range of K/V columns at a
    time.  Returns (pieces int32[P, 4] = (window, first block, end block, slot
    or -1), splits int32[S, 4] = (window, first slot, pieces, 0), number of
    slots, chunk_starts int64[C + 1]): the pieces of chunk c are rows
    chunk_starts[c] ... chunk_starts[c + 1] - 1; a window without blocks is
    one empty piece in chunk 0.  A window's pieces own consecutive slots in
    column order (merged in that order)."""
    off = np.asarray(window_offsets, dtype=np.int64)
    cols = np.asarray(block_cols, dtype=np.int64)
    order = np.asarray(order, dtype=np.int64)
    if col_cuts is None:
        if chunk_cols < 1:
            raise ValueError("chunk_cols must be >= 1")
        n_cols = off.shape[0] - 1
        col_cuts = np.arange(0, n_cols + chunk_cols, chunk_cols, dtype=np.int64)
        if col_cuts.shape[0] < 2:
            col_cuts = np.array([0, max(chunk_cols, 1)], np.int64)
    col_cuts = np.asarray(col_cuts, dtype=np.int64)
    if col_cuts.ndim != 1 or col_cuts.shape[0] < 2 or col_cuts[0] != 0 or np.any(np.diff(col_cuts) < 0):
        raise ValueError("col_cuts must be ascending boundaries starting at 0")
    n_chunks = col_cuts.shape[0] - 1
    starts, ends = off[order], off[order + 1]
    counts = ends - starts
    keep = counts > 0
    empty_windows = order[~keep]
    n_blocks = int(counts.sum())
    item = np.repeat(np.arange(order.shape[0]), counts)           # listed index of every block
    blk = np.arange(n_blocks) - np.repeat(np.cumsum(counts) - counts, counts) + np.repeat(starts, counts)
    chunk = (np.searchsorted(col_cuts, cols[blk], side="right") - 1) if n_blocks else np.zeros(0, np.int64)
    if n_blocks and (chunk.min() < 0 or chunk.max() >= n_chunks):
        raise ValueError("col_cuts do not cover every block column")
    first_of_item = np.ones(n_blocks, bool)
    if n_blocks:
        first_of_item[1:] = item[1:] != item[:-1]
    run_start = first_of_item.copy()
    if n_blocks:
        run_start[1:] |= chunk[1:] != chunk[:-1]
    idx = np.arange(n_blocks)
    if max_blocks and max_blocks > 0 and n_blocks:
        run_begin = np.maximum.accumulate(np.where(run_start, idx, 0))
        cut = run_start | ((idx - run_begin) % max_blocks == 0)
    else:
        cut = run_start
    p_start = np.flatnonzero(cut)
    p_end = np.append(p_start[1:], n_blocks)
    p_item = item[p_start]
    p_chunk = chunk[p_start]
    per_item = np.bincount(p_item, minlength=order.shape[0])
    split = per_item > 1
    # slots: consecutive per split window, in the window's column order
    slot_base = np.cumsum(np.where(split, per_item, 0)) - np.where(split, per_item, 0)
    rank_in_item = np.arange(p_start.shape[0]) - (np.cumsum(per_item) - per_item)[p_item]
    p_slot = np.where(split[p_item], slot_base[p_item] + rank_in_item, -1)
    pieces = np.stack([order[p_item], blk[p_start], blk[p_end - 1] + 1, p_slot], axis=1).reshape(-1, 4)
    if empty_windows.size:  # windows without blocks still write zero rows (chunk 0)
        z = np.stack([empty_windows, off[empty_windows], off[empty_windows], -np.ones_like(empty_windows)], axis=1)
        pieces = np.concatenate([pieces, z])
        p_chunk = np.concatenate([p_chunk, np.zeros(empty_windows.shape[0], np.int64)])
    sort = np.argsort(p_chunk, kind="stable")
    pieces = pieces[sort]
    chunk_starts = np.zeros(n_chunks + 1, np.int64)
    np.cumsum(np.bincount(p_chunk, minlength=n_chunks)[:n_chunks], out=chunk_starts[1:])
    s_items = np.flatnonzero(split)
    splits = np.stack([order[s_items], slot_base[s_items], per_item[s_items], np.zeros_like(s_items)], axis=1)
    n_slots = int(per_item[split].sum())
    return (pieces.astype(np.int32).reshape(-1, 4), splits.astype(np.int32).reshape(-1, 4), n_slots,
            chunk_starts)


def make_chunked_plan(fmt: BlockSparseFormat, heads: int, head_dim: int, order: Optional[torch.Tensor] = None,
                      chunk_cols: Optional[int] = None, max_blocks: int = 0, l2_fraction: float = 0.5) -> ForwardPlan:
    """A plan that sweeps the block columns in chunks (column_chunk_pieces),
    uploaded with f3s_load_plan.  chunk_cols defaults to the number of block
    columns whose K and V tiles (16 rows x heads x head_dim x 2 B each) fill
    `l2_fraction` of the device's L2.  Partial states take 64 * heads *
    (head_dim + 2) bytes per piece of a split window."""
    lib = _lib.load()
    device = fmt.window_offsets.device
    if order is None:
        order = generate_balanced_window_order(fmt)
    off, cols = fmt.to_host()
    order_h = order.cpu().numpy().astype(np.int64)
    if chunk_cols is None:
        l2 = torch.cuda.get_device_properties(device).L2_cache_size
        chunk_cols = max(1, int(l2 * l2_fraction) // (16 * heads * head_dim * 2 * 2))
    pieces, splits, n_slots, _ = column_chunk_pieces(off, cols, order_h, int(chunk_cols), int(max_blocks))
    return load_plan(fmt, pieces, splits, n_slots, heads, head_dim, off_host=off, max_blocks=int(max_blocks))


def load_plan(fmt: BlockSparseFormat, pieces: np.ndarray, splits: np.ndarray, n_slots: int, heads: int,
              head_dim: int, off_host: Optional[np.ndarray] = None, max_blocks: int = 0,
              piece_ranges=None) -> ForwardPlan:
    """Upload a host-built plan (f3s_load_plan, validated on the host)."""
    lib = _lib.load()
    device = fmt.window_offsets.device
    off = fmt.window_offsets.cpu().numpy() if off_host is None else off_host
    pieces = np.ascontiguousarray(pieces, dtype=np.int32).reshape(-1, 4)
    splits = np.ascontiguousarray(splits, dtype=np.int32).reshape(-1, 4)
    size = lib.f3s_plan_size_for(pieces.shape[0], splits.shape[0], int(n_slots), heads, head_dim)
    if size == 0:
        raise ValueError("unsupported plan parameters")
    buf = torch.empty(size, dtype=torch.uint8, device=device)
    off32 = np.ascontiguousarray(off.astype(np.int32))
    with torch.cuda.device(device):
        st = lib.f3s_load_plan(pieces.ctypes.data, pieces.shape[0], splits.ctypes.data if splits.size else None,
                               splits.shape[0], int(n_slots), off32.ctypes.data, fmt.num_row_windows, heads,
                               head_dim, _ptr(buf), size, _stream_ptr(device))
    check(st, "f3s_load_plan")
    return ForwardPlan(buf, heads, head_dim, int(max_blocks), piece_ranges)


def make_sweep_plan(fmt: BlockSparseFormat, heads: int, head_dim: int, order: Optional[torch.Tensor] = None,
                    chunk_cols: Optional[int] = None, l2_fraction: float = 1.0, window_range=None) -> ForwardPlan:
    """A sweep plan (f3s_load_sweep_plan): every listed window cut where its
    block columns cross a multiple of `chunk_cols`, the pieces ordered chunk by
    chunk (windows in `order` within a chunk), so all SMs read one range of
    K / V at a time and the L2 serves the rest of the chunk's reads; a window
    carries its running softmax state from piece to piece (no partial state
    per piece, no merge).  chunk_cols defaults to the block columns whose K
    and V tiles fill `l2_fraction` of the device's L2.  window_range: the
    slab (lo, hi) whose windows `order` lists (default all windows)."""
    lib = _lib.load()
    device = fmt.window_offsets.device
    if order is None:
        order = generate_balanced_window_order(fmt)
    off, cols = fmt.to_host()
    order_h = order.cpu().numpy().astype(np.int64)
    if chunk_cols is None:
        l2 = torch.cuda.get_device_properties(device).L2_cache_size
        chunk_cols = max(1, int(l2 * l2_fraction) // (16 * heads * head_dim * 2 * 2))
    pieces, _, _, _ = column_chunk_pieces(off, cols, order_h, int(chunk_cols), 0)
    lo, hi = window_range if window_range is not None else (0, fmt.num_row_windows)
    pieces = np.ascontiguousarray(pieces, dtype=np.int32)
    size = lib.f3s_sweep_plan_size(pieces.shape[0], hi - lo, heads, head_dim)
    if size == 0:
        raise ValueError("unsupported plan parameters")
    buf = torch.empty(size, dtype=torch.uint8, device=device)
    off32 = np.ascontiguousarray(off.astype(np.int32))
    with torch.cuda.device(device):
        st = lib.f3s_load_sweep_plan(pieces.ctypes.data, pieces.shape[0], off32.ctypes.data, fmt.num_row_windows,
                                     lo, hi - lo, heads, head_dim, _ptr(buf), size, _stream_ptr(device))
    check(st, "f3s_load_sweep_plan")
    return ForwardPlan(buf, heads, head_dim, int(chunk_cols), sweep=True)


def column_slices(num_nodes: int, parts: int):
    """K / V cut into `parts` slices of whole block columns: boundaries
    col_cuts[0] = 0 < ... < col_cuts[parts] = ceil(num_nodes / 16) (equal
    sizes up to one block column), and each slice's node rows [r0, r1)."""
    nrw = (num_nodes + 15) // 16
    cuts = np.array([(nrw * j) // parts for j in range(parts + 1)], np.int64)
    rows = [(min(16 * int(a), num_nodes), min(16 * int(b), num_nodes)) for a, b in zip(cuts[:-1], cuts[1:])]
    return cuts, rows


def make_sliced_plan(fmt: BlockSparseFormat, heads: int, head_dim: int, col_cuts, order: Optional[torch.Tensor] = None,
                     max_blocks: int = 0) -> ForwardPlan:
    """A plan for K / V held in slices of block columns (col_cuts, e.g. from
    column_slices): every listed window is cut at the slice boundaries, and
    the pieces of slice j are plan.piece_ranges[j] -- run them with
    forward_pieces(..., kv_col_base=col_cuts[j]) on that slice's K / V rows,
    in any slice order, then plan_merge once."""
    device = fmt.window_offsets.device
    if order is None:
        order = generate_balanced_window_order(fmt)
    off, cols = fmt.to_host()
    order_h = order.cpu().numpy().astype(np.int64)
    pieces, splits, n_slots, starts = column_chunk_pieces(off, cols, order_h, max_blocks=int(max_blocks),
                                                          col_cuts=col_cuts)
    ranges = [(int(a), int(b)) for a, b in zip(starts[:-1], starts[1:])]
    return load_plan(fmt, pieces, splits, n_slots, heads, head_dim, off_host=off, max_blocks=int(max_blocks),
                     piece_ranges=ranges)


_OUT_DTYPES = {torch.float32: _lib.F3S_OUT_F32, torch.float16: _lib.F3S_OUT_F16,
               torch.bfloat16: _lib.F3S_OUT_BF16}


def fused3s_forward(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, fmt: BlockSparseFormat,
                    order: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                    q_window_base: int = 0, check_status: bool = False,
                    block_hints: Optional[torch.Tensor] = None, plan: Optional[ForwardPlan] = None,
                    out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """O = block-sparse softmax(Q K^T) V, fused (the fused3s_v2 path).

    Q: fp16 [q_rows, H, d] (or [q_rows, d] for one head) holding rows
       16*q_window_base ... of the full Q;  K, V: fp16 [N, H, d] (or [N, d]).
    order: int32 window ids to compute (default: every window of the slab in
       the balanced order).  Returns fp32 O shaped like Q; rows of the listed
       windows are written in full (zeros for windows with no block).
    check_status: synchronise and raise if a kernel recorded an error.
    block_hints: optional uint8[num_blocks] from block_hints() (speed only).
    plan: optional ForwardPlan from make_plan(); it then lists the windows
       (order is ignored) and heavy windows run as several pieces.
    out_dtype: element type of O when `out` is not given: float32 (as
       computed), or float16 / bfloat16 (the fp32 result rounded to nearest)."""
    if plan is not None and (plan.heads, plan.head_dim) != (_as_nhd(Q).shape[1], _as_nhd(Q).shape[2]):
        raise ValueError("plan was made for other heads / head_dim")
    if block_hints is not None and (block_hints.dtype != torch.uint8 or block_hints.numel() < fmt.num_blocks):
        raise ValueError("block_hints must be uint8 with one entry per active block")
    lib = _lib.load()
    _check_features(Q, K, V)
    q3, k3 = _as_nhd(Q), _as_nhd(K)
    q_rows, heads, head_dim = q3.shape
    num_nodes = k3.shape[0]
    if k3.shape[1:] != (heads, head_dim):
        raise ValueError("Q, K, V must agree on heads and head_dim")
    if num_nodes != fmt.num_nodes:
        raise ValueError("K/V rows must equal the graph's num_nodes")
    device = Q.device
    if plan is not None:
        order = torch.zeros(1, dtype=torch.int32, device=device)  # unused: the plan lists the windows
    elif order is None:
        if q_window_base == 0 and q_rows == num_nodes:
            order = generate_balanced_window_order(fmt)
        else:
            order = torch.arange(q_window_base, q_window_base + (q_rows + 15) // 16, dtype=torch.int32,
                                 device=device)
    order = order.to(device=device, dtype=torch.int32).contiguous()
    if out is None:
        out = torch.empty(Q.shape, dtype=out_dtype, device=device)
    elif out.shape != Q.shape or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor shaped like Q")
    if out.dtype not in _OUT_DTYPES:
        raise ValueError("O must be float32, float16 or bfloat16")
    ws_bytes = (lib.f3s_sweep_workspace_size(q_rows, heads) if plan is not None and plan.sweep
                else lib.f3s_forward_workspace_size())
    ws = _WS.get(device, "forward", ws_bytes)
    with torch.cuda.device(device):
        st = lib.f3s_forward_ex(_ptr(Q), _ptr(K), _ptr(V), _ptr(out), _OUT_DTYPES[out.dtype],
                                _ptr(fmt.window_offsets), fmt.cols_ptr, _ptr(order), _ptr(block_hints),
                                None if plan is None else _ptr(plan.buffer), int(order.numel()), num_nodes, heads,
                                head_dim, q_window_base, q_rows, _ptr(ws), ws.numel(), _stream_ptr(device))
        check(st, "f3s_forward_ex")
        if check_status:
            check(lib.f3s_workspace_status(_ptr(ws), _stream_ptr(device)), "f3s_forward (device)")
    return out


def forward_pieces(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, fmt: BlockSparseFormat, plan: ForwardPlan,
                   out: torch.Tensor, piece_begin: int = 0, piece_end: int = -1, kv_col_base: int = 0,
                   q_window_base: int = 0, block_hints: Optional[torch.Tensor] = None,
                   check_status: bool = False) -> torch.Tensor:
    """Pieces [piece_begin, piece_end) of `plan` (f3s_forward_pieces), with
    K / V holding only the graph's rows 16 * kv_col_base ... (K.shape[0]
    rows): windows of one piece get their O rows, split windows' pieces
    leave partial states in the plan for plan_merge.  No merge here."""
    lib = _lib.load()
    _check_features(Q, K, V)
    q3, k3 = _as_nhd(Q), _as_nhd(K)
    q_rows, heads, head_dim = q3.shape
    if k3.shape[1:] != (heads, head_dim) or (plan.heads, plan.head_dim) != (heads, head_dim):
        raise ValueError("Q, K, V and the plan must agree on heads and head_dim")
    if out.shape != Q.shape or not out.is_contiguous() or out.dtype not in _OUT_DTYPES:
        raise ValueError("out must be a contiguous float32/float16/bfloat16 tensor shaped like Q")
    device = Q.device
    ws = _WS.get(device, "forward", lib.f3s_forward_workspace_size())
    with torch.cuda.device(device):
        st = lib.f3s_forward_pieces(_ptr(Q), _ptr(K), _ptr(V), _ptr(out), _OUT_DTYPES[out.dtype],
                                    _ptr(fmt.window_offsets), fmt.cols_ptr, _ptr(block_hints), _ptr(plan.buffer),
                                    int(piece_begin), int(piece_end), int(kv_col_base), int(k3.shape[0]),
                                    fmt.num_nodes, heads, head_dim, int(q_window_base), q_rows, _ptr(ws),
                                    ws.numel(), _stream_ptr(device))
        check(st, "f3s_forward_pieces")
        if check_status:
            check(lib.f3s_workspace_status(_ptr(ws), _stream_ptr(device)), "f3s_forward_pieces (device)")
    return out


def plan_merge(plan: ForwardPlan, out: torch.Tensor, num_nodes: int, q_window_base: int = 0) -> torch.Tensor:
    """Writes the O rows of the plan's split windows from their partial
    states (f3s_plan_merge), after every piece ran."""
    lib = _lib.load()
    o3 = _as_nhd(out)
    if out.dtype not in _OUT_DTYPES or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32/float16/bfloat16 tensor")
    device = out.device
    with torch.cuda.device(device):
        st = lib.f3s_plan_merge(_ptr(plan.buffer), _ptr(out), _OUT_DTYPES[out.dtype], int(num_nodes), plan.heads,
                                plan.head_dim, int(q_window_base), o3.shape[0], _stream_ptr(device))
    check(st, "f3s_plan_merge")
    return out


def set_forward_sm_limit(max_ctas: int, device=None) -> None:
    """At most max_ctas persistent CTAs per forward launch on `device` from
    now on (0: one per SM); leaves SMs to a kernel that runs beside the
    forward, e.g. an NCCL all-gather on another stream."""
    device = _default_device(device)
    with torch.cuda.device(device):
        check(_lib.load().f3s_set_forward_sm_limit(int(max_ctas)), "f3s_set_forward_sm_limit")


def forward_workspace(device=None) -> torch.Tensor:
    """The workspace fused3s_forward uses on the current stream of `device`."""
    device = _default_device(device)
    return _WS.get(device, "forward", _lib.load().f3s_forward_workspace_size())


def workspace_status(ws: torch.Tensor) -> int:
    """Synchronise and return (and clear) the first error a kernel recorded in ws."""
    return _lib.load().f3s_workspace_status(_ptr(ws), _stream_ptr(ws.device))


def f3s_1tb1rw_kernel(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, O_out: torch.Tensor,
                      window_offsets: torch.Tensor, block_col_indices: torch.Tensor,
                      window_order: torch.Tensor, num_row_windows: int, feat_dim: int) -> None:
    """Drop-in for the reference kernel launch <<<nrw, dim3(32,4)>>> (src/fused3s_v2.cu:81-90):
    same arguments, buffers with num_row_windows*16 rows, every row treated as
    a node (no masking of padded columns, like the reference v2 kernel)."""
    lib = _lib.load()
    rows = num_row_windows * 16
    for name, t, dt in (("Q", Q, torch.float16), ("K", K, torch.float16), ("V", V, torch.float16),
                        ("O_out", O_out, torch.float32)):
        if t.dtype != dt or not t.is_contiguous() or t.numel() < rows * feat_dim:
            raise ValueError(f"{name}: expected contiguous {dt} with {rows}x{feat_dim} elements")
    device = Q.device
    with torch.cuda.device(device):
        st = lib.f3s_1tb1rw_launch(_ptr(Q), _ptr(K), _ptr(V), _ptr(O_out), _ptr(window_offsets),
                                   _ptr(block_col_indices), _ptr(window_order), num_row_windows, feat_dim,
                                   _stream_ptr(device))
    check(st, "f3s_1tb1rw_launch")


def float2half(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> fp16 round-to-nearest on the GPU (tests/test_fused_3s_v2.cu:61-64)."""
    lib = _lib.load()
    if x.dtype != torch.float32 or x.device.type != "cuda":
        raise TypeError("float2half expects a CUDA float32 tensor")
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=torch.float16, device=x.device)
    with torch.cuda.device(x.device):
        st = lib.f3s_half_from_float(_ptr(x), _ptr(out), x.numel(), _stream_ptr(x.device))
    check(st, "f3s_half_from_float")
    return out
