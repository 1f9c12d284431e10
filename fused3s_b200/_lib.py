"""ctypes binding of libfused3s.so (the C ABI declared in include/fused3s.h).

The library is the only compute path: if it is missing or fails to load,
every entry point raises.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("FUSED3S_LIB", _PKG / "libfused3s.so"))

F3S_SUCCESS = 0
F3S_ERR_INVALID_VALUE = 1
F3S_ERR_UNSUPPORTED = 2
F3S_ERR_BAD_CSR = 3
F3S_ERR_WORKSPACE = 4
F3S_ERR_CUDA = 5
F3S_ERR_TIMEOUT = 6
F3S_ERR_BAD_FORMAT = 7
F3S_ERR_TOO_LARGE = 8

F3S_IPC_HANDLE_BYTES = 64

F3S_OUT_F32 = 0
F3S_OUT_F16 = 1
F3S_OUT_BF16 = 2

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_U64 = ctypes.c_uint64

# name -> (restype, argtypes); mirrors include/fused3s.h one to one
SIGNATURES = {
    "f3s_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "f3s_version": (ctypes.c_int, []),
    "f3s_last_cuda_error": (ctypes.c_int, []),
    "f3s_set_forward_sm_limit": (ctypes.c_int, [_I32]),
    "f3s_workspace_status": (ctypes.c_int, [_P, _P]),
    "f3s_convert_workspace_size": (_SZ, [_I32, _I64]),
    "f3s_convert": (ctypes.c_int, [_P, _P, _I32, _I64, _P, _P, _P, _SZ, ctypes.POINTER(_I64), _P]),
    "f3s_convert_noalloc": (ctypes.c_int, [_P, _P, _I32, _I64, _P, _P, ctypes.POINTER(_I64), _P]),
    "f3s_window_order_workspace_size": (_SZ, [_I32]),
    "f3s_window_order": (ctypes.c_int, [_P, _I32, _P, _P, _SZ, _P]),
    "f3s_forward_workspace_size": (_SZ, []),
    "f3s_forward": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _P,
                                   _SZ, _P]),
    "f3s_forward_ex": (ctypes.c_int, [_P, _P, _P, _P, _I32, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
                                      _P, _SZ, _P]),
    "f3s_parse_int32_workspace_size": (_SZ, [_I64]),
    "f3s_parse_int32": (ctypes.c_int, [_P, _I64, _P, _I64, ctypes.POINTER(ctypes.c_int64), _P, _SZ, _P]),
    "f3s_peer_alloc": (ctypes.c_int, [_SZ, ctypes.POINTER(ctypes.c_void_p), _P]),
    "f3s_peer_open": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "f3s_peer_close": (ctypes.c_int, [_P]),
    "f3s_peer_free": (ctypes.c_int, [_P]),
    "f3s_peer_copy": (ctypes.c_int, [_P, _P, _SZ, _P]),
    "f3s_plan_size": (_SZ, [_I32, _I64, _I32, _I32, _I32]),
    "f3s_plan_size_for": (_SZ, [_I32, _I32, _I32, _I32, _I32]),
    "f3s_load_plan": (ctypes.c_int, [_P, _I32, _P, _I32, _I32, _P, _I32, _I32, _I32, _P, _SZ, _P]),
    "f3s_make_plan": (ctypes.c_int, [_P, _P, _I32, _I64, _I32, _I32, _I32, _P, _SZ, _P]),
    "f3s_forward_pieces": (ctypes.c_int, [_P, _P, _P, _P, _I32, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
                                          _I32, _I32, _I32, _P, _SZ, _P]),
    "f3s_plan_merge": (ctypes.c_int, [_P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _P]),
    "f3s_sweep_plan_size": (_SZ, [_I32, _I32, _I32, _I32]),
    "f3s_sweep_workspace_size": (_SZ, [_I32, _I32]),
    "f3s_load_sweep_plan": (ctypes.c_int, [_P, _I32, _P, _I32, _I32, _I32, _I32, _I32, _P, _SZ, _P]),
    "f3s_block_hints_workspace_size": (_SZ, [_I32]),
    "f3s_block_hints": (ctypes.c_int, [_P, _P, _P, _I32, _I32, _I64, _I64, _P, _P, _SZ, _P]),
    "f3s_1tb1rw_launch": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _P]),
    "f3s_half_from_float": (ctypes.c_int, [_P, _P, _I64, _P]),
    "f3s_selftest_wait_timeout": (ctypes.c_int, [_U64, _P, _SZ, _P]),
    "f3s_probe_mma_sync": (ctypes.c_int, [_I32, _I32, ctypes.POINTER(ctypes.c_double), _P]),
}

_lib = None


class Fused3SError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        msg = status_string(status) if _lib is not None else str(status)
        if status == F3S_ERR_CUDA and _lib is not None:
            msg += f" (cudaError {_lib.f3s_last_cuda_error()})"
        super().__init__(f"{where}: {msg}")


def load():
    """Load libfused3s.so (once) and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m fused3s_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def status_string(status: int) -> str:
    return load().f3s_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status != F3S_SUCCESS:
        raise Fused3SError(status, where)
