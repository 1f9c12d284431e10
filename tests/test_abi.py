"""The C-ABI library loads on a machine without a GPU and exports exactly
what include/fused3s.h declares.  No compute call is made here."""
import ctypes
import re

import numpy as np
import pytest

from conftest import ROOT
from fused3s_b200 import _lib


def declared_functions():
    text = (ROOT / "include" / "fused3s.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(f3s_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_surface():
    names = declared_functions()
    for must in ("f3s_convert", "f3s_window_order", "f3s_forward", "f3s_1tb1rw_launch",
                 "f3s_workspace_status", "f3s_half_from_float"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)


def test_python_binding_covers_the_header():
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_host_only_queries(lib):
    assert lib.f3s_version() >= 10000
    assert lib.f3s_forward_workspace_size() == 256
    assert lib.f3s_convert_workspace_size(2708, 13264) >= 256 + 4 * 13264
    assert lib.f3s_convert_workspace_size(-1, 0) == 0
    assert lib.f3s_window_order_workspace_size(1 << 20) > 4 * (1 << 20) * 4
    for code in range(0, 9):
        s = lib.f3s_status_string(code).decode()
        assert s.startswith("F3S_")
    assert "UNKNOWN" in lib.f3s_status_string(99).decode()


def test_invalid_arguments_are_rejected_without_touching_the_gpu(lib):
    # validated on the host before any CUDA call
    assert lib.f3s_forward(None, None, None, None, None, None, None, None, None, 1, 10, 1, 96, 0, 10, None, 0,
                           None) == _lib.F3S_ERR_UNSUPPORTED
    assert lib.f3s_forward(None, None, None, None, None, None, None, None, None, 1, 10, 1, 64, 0, 10, None, 0,
                           None) == _lib.F3S_ERR_INVALID_VALUE
    assert lib.f3s_convert(None, None, -1, 0, None, None, None, 0, None, None) == _lib.F3S_ERR_INVALID_VALUE
    assert lib.f3s_window_order(None, -3, None, None, 0, None) == _lib.F3S_ERR_INVALID_VALUE
    assert lib.f3s_half_from_float(None, None, -1, None) == _lib.F3S_ERR_INVALID_VALUE
    n = _lib.ctypes.c_int64(0)
    assert lib.f3s_parse_int32(None, -1, None, 0, n, 256, 256, None) == _lib.F3S_ERR_INVALID_VALUE
    assert lib.f3s_parse_int32(None, 1 << 33, None, 0, n, 256, 256, None) == _lib.F3S_ERR_TOO_LARGE
    assert lib.f3s_parse_int32(None, 0, None, 0, n, 256, 256, None) == 0 and n.value == 0
    assert lib.f3s_peer_copy(None, None, 16, None) == _lib.F3S_ERR_INVALID_VALUE
    assert lib.f3s_forward_ex(None, None, None, None, 7, None, None, None, None, None, 1, 10, 1, 64, 0, 10, 256,
                              256, None) == _lib.F3S_ERR_INVALID_VALUE


def test_product_package_does_not_reference_the_oracle():
    """The shipped package never imports or loads the oracle."""
    pkg = ROOT / "fused3s_b200"
    for path in list(pkg.glob("*.py")) + list((pkg / "csrc").glob("*")):
        text = path.read_text()
        assert "import oracle" not in text and "liboracle" not in text and "libf3s_ref" not in text, path


def test_text_pieces_cut_at_separators():
    """Host side of the GPU text reader: pieces of at most `limit` bytes that
    end after a separator cover the text, and no number is split."""
    from fused3s_b200.api import text_pieces
    rng = np.random.default_rng(0)
    vals = rng.integers(0, 10**9, 5000)
    text = np.frombuffer(("\n".join(str(v) for v in vals) + "\n").encode(), dtype=np.uint8)
    for limit in (16, 64, 1000, len(text), len(text) + 5):
        cuts = text_pieces(text, limit)
        assert cuts[0][0] == 0 and cuts[-1][1] == len(text)
        assert all(b - a <= limit for a, b in cuts)
        assert all(b == c for (_, b), (c, _) in zip(cuts[:-1], cuts[1:]))
        joined = [int(x) for a, b in cuts for x in bytes(text[a:b]).split()]
        assert np.array_equal(joined, vals)
    with pytest.raises(ValueError):
        text_pieces(np.frombuffer(b"123456789 1", dtype=np.uint8), 4)


def test_c_usage_compiles_as_plain_c():
    """The documented C call sequence compiles against include/fused3s.h with
    a C compiler (the header stays plain C, every call matches its
    declaration)."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    r = subprocess.run([gcc, "-std=c11", "-Wall", "-Werror", "-fsyntax-only", f"-I{ROOT / 'include'}",
                        str(ROOT / "tests" / "cpp" / "c_abi_usage.c")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
