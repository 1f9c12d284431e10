"""f3s_load_plan checks a caller-built plan on the host before anything is
copied: indices in range, every listed window's blocks covered exactly once,
slot ownership consistent with the split records.  An inconsistent plan is
rejected with F3S_ERR_BAD_FORMAT (no GPU needed: the check runs before the
first CUDA call; a consistent plan gets past it, so on a machine without a
GPU it fails later, at the copy, with another code)."""
import numpy as np

from fused3s_b200 import _lib

# 4 windows: w0 has blocks [0, 5), w1 [5, 5) (none), w2 [5, 9), w3 [9, 12)
OFF = np.array([0, 5, 5, 9, 12], np.int32)
NRW = 4


def load(lib, pieces, splits, n_slots):
    p = np.ascontiguousarray(np.asarray(pieces, np.int32).reshape(-1, 4))
    s = np.ascontiguousarray(np.asarray(splits, np.int32).reshape(-1, 4))
    size = lib.f3s_plan_size_for(p.shape[0], s.shape[0], n_slots, 1, 64)
    fake_plan = 1 << 20  # 256-byte aligned; never dereferenced on the host
    return lib.f3s_load_plan(p.ctypes.data, p.shape[0], s.ctypes.data if s.size else None, s.shape[0], n_slots,
                             OFF.ctypes.data, NRW, 1, 64, fake_plan, size, None)


VALID = (
    # w0 split in two (slots 0, 1), w1 empty, w2 whole, w3 split in three (slots 2..4)
    [(0, 0, 3, 0), (1, 5, 5, -1), (2, 5, 9, -1), (3, 9, 10, 2), (0, 3, 5, 1), (3, 10, 11, 3), (3, 11, 12, 4)],
    [(0, 0, 2, 0), (3, 2, 3, 0)],
    5,
)


def test_consistent_plans_pass_the_host_check(lib):
    assert load(lib, *VALID) != _lib.F3S_ERR_BAD_FORMAT
    # a subset of the windows is a valid plan too
    assert load(lib, [(2, 5, 9, -1)], [], 0) != _lib.F3S_ERR_BAD_FORMAT


def test_inconsistent_plans_are_rejected(lib):
    pieces, splits, n = VALID

    def with_piece(i, new):
        p = list(pieces)
        p[i] = new
        return p

    cases = {
        "overlap": (with_piece(4, (0, 2, 5, 1)), splits, n),
        "gap": (with_piece(4, (0, 4, 5, 1)), splits, n),
        "missing tail": (with_piece(2, (2, 5, 8, -1)), splits, n),
        "orphan slot (another window's)": (with_piece(4, (0, 3, 5, 2)), splits, n),
        "slot used twice": (with_piece(4, (0, 3, 5, 0)), splits, n),
        "unsplit piece of a split window": (with_piece(4, (0, 3, 5, -1)), splits, n),
        "split record count disagrees": (pieces, [(0, 0, 2, 0), (3, 2, 2, 0)], n),
        "single piece with a slot": (with_piece(2, (2, 5, 9, 4)), splits, n),
        "window split but no record": (pieces, [(3, 2, 3, 0)], n),
        "records share a slot": (pieces, [(0, 0, 2, 0), (3, 1, 3, 0)], n),
        "two records for one window": (pieces, [(0, 0, 2, 0), (3, 2, 3, 0), (0, 0, 2, 0)], n),
        "empty piece in a window with blocks": (pieces + [(2, 9, 9, -1)], splits, n),
        "window id out of range": (with_piece(1, (4, 5, 5, -1)), splits, n),
        "slot out of range": (with_piece(4, (0, 3, 5, 5)), splits, n),
        "record slot never used": (pieces, [(0, 0, 2, 0), (3, 2, 3, 0)], n + 1),
    }
    for name, (p, s, k) in cases.items():
        if name == "record slot never used":
            s = s + [(1, 5, 1, 0)]  # w1 has a record but its single empty piece has slot -1
        assert load(lib, p, s, k) == _lib.F3S_ERR_BAD_FORMAT, name


def load_sweep(lib, pieces, q_window_base=0, q_windows=NRW):
    p = np.ascontiguousarray(np.asarray(pieces, np.int32).reshape(-1, 4))
    size = lib.f3s_sweep_plan_size(p.shape[0], q_windows, 1, 64)
    fake_plan = 1 << 20
    return lib.f3s_load_sweep_plan(p.ctypes.data, p.shape[0], OFF.ctypes.data, NRW, q_window_base, q_windows, 1,
                                   64, fake_plan, size, None)


def test_sweep_plans_are_validated(lib):
    """Sweep plans (f3s_load_sweep_plan): a window's pieces in ascending block
    order covering its blocks once, windows inside the slab."""
    good = [(0, 0, 2, 0), (2, 5, 9, 0), (0, 2, 5, 0), (1, 5, 5, 0), (3, 9, 12, 0)]
    assert load_sweep(lib, good) != _lib.F3S_ERR_BAD_FORMAT
    assert load_sweep(lib, [(2, 5, 7, 0), (3, 9, 12, 0), (2, 7, 9, 0)], 2, 2) != _lib.F3S_ERR_BAD_FORMAT
    bad = {
        "out of column order": [(0, 2, 5, 0), (0, 0, 2, 0)],
        "overlap": [(0, 0, 3, 0), (0, 2, 5, 0)],
        "gap": [(0, 0, 2, 0), (0, 3, 5, 0)],
        "not covered": [(0, 0, 2, 0)],
        "empty piece of a window with blocks": [(0, 0, 0, 0), (0, 0, 5, 0)],
        "window outside the slab": [(3, 9, 12, 0)],
        "piece beyond its window": [(2, 5, 10, 0)],
    }
    for name, pieces in bad.items():
        qb, qw = (0, 3) if name == "window outside the slab" else (0, NRW)
        assert load_sweep(lib, pieces, qb, qw) == _lib.F3S_ERR_BAD_FORMAT, name
