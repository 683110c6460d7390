"""ctypes binding of the C ABI in include/gemm_sm100.h (libgemm_sm100.so).

The shared library is built in-tree by ``infinite-dreams_b200/build.py``.  If
it is missing this module raises at import: there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import List, Tuple

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libgemm_sm100.so"

GEMM_OK = 0
GEMM_ERR_INVALID_ARG = 1
GEMM_ERR_BAD_CFG = 2
GEMM_ERR_WORKSPACE = 3
GEMM_ERR_CUDA = 4
GEMM_ERR_UNSUPPORTED = 5
GEMM_ERR_DEVICE_TIMEOUT = 6

GEMM_MAX_PEERS = 7
GEMM_IPC_HANDLE_BYTES = 64

GEMM_ACT_NONE = 0
GEMM_ACT_RELU = 1
GEMM_ACT_GELU = 2
ACTIVATIONS = {"none": GEMM_ACT_NONE, "relu": GEMM_ACT_RELU, "gelu": GEMM_ACT_GELU}

# (name, restype, argtypes) of every exported entry point.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SIG = [
    ("gemm_num_cfgs", ctypes.c_int, []),
    ("gemm_cfg_num_cols", ctypes.c_int, []),
    ("gemm_cfg_col_name", ctypes.c_char_p, [ctypes.c_int]),
    ("gemm_cfg_row", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    ("gemm_cfg_find", ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    ("gemm_workspace_bytes", ctypes.c_size_t, [_P, _P, _I64, _I64, _I64, _I64, _I64, ctypes.c_int]),
    ("gemm_workspace_counter_bytes", ctypes.c_size_t, []),
    ("gemm_launch", ctypes.c_int,
     [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, ctypes.c_int, _P, ctypes.c_size_t, _P]),
    ("gemm_launch_knobs", ctypes.c_int,
     [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, ctypes.POINTER(ctypes.c_int), ctypes.c_int, _P,
      ctypes.c_size_t, _P]),
    ("gemm_launch_noalloc", ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, ctypes.c_int, _P]),
    ("gemm_launch_ex", ctypes.c_int,
     [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
      _P, _I64, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_size_t, _P]),
    ("gemm_workspace_bytes_ex", ctypes.c_size_t,
     [_P, _P, _I64, _I64, _I64, _I64, _I64, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    ("gemm_launch_gather", ctypes.c_int,
     [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
      _P, ctypes.c_size_t, _P]),
    ("gemm_launch_multicast", ctypes.c_int,
     [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, ctypes.c_int, _P, ctypes.c_size_t, _P]),
    ("gemm_ipc_export", ctypes.c_int, [_P, _P, ctypes.POINTER(ctypes.c_int64)]),
    ("gemm_ipc_import", ctypes.c_int, [_P, _I64, ctypes.POINTER(ctypes.c_void_p)]),
    ("gemm_ipc_close", ctypes.c_int, [_P]),
    ("gemm_default_cfg", ctypes.c_int, [_I64, _I64, _I64]),
    ("gemm_device_error", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    ("gemm_selftest_wait_timeout", ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    ("gemm_last_error", ctypes.c_char_p, []),
    ("gemm_status_string", ctypes.c_char_p, [ctypes.c_int]),
]


class GemmError(RuntimeError):
    """A non-OK status from the kernel bank's C ABI."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def _load() -> ctypes.CDLL:
    path = Path(os.environ.get("INFINITE_DREAMS_GEMM_LIB", str(LIB_PATH)))
    if not path.exists():
        raise ImportError(
            f"libgemm_sm100.so not found at {path}; build it with "
            "`python infinite-dreams_b200/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(str(path))
    for name, res, args in _SIG:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def symbols() -> List[str]:
    return [s[0] for s in _SIG]


def check(status: int, what: str = "gemm") -> None:
    if status != GEMM_OK:
        msg = lib.gemm_last_error().decode(errors="replace")
        name = lib.gemm_status_string(status).decode()
        raise GemmError(status, f"{what}: {name}: {msg}")


def menu() -> Tuple[List[str], List[Tuple[int, ...]]]:
    ncol = lib.gemm_cfg_num_cols()
    cols = [lib.gemm_cfg_col_name(i).decode() for i in range(ncol)]
    rows = []
    buf = (ctypes.c_int * ncol)()
    for i in range(lib.gemm_num_cfgs()):
        check(lib.gemm_cfg_row(i, buf, ncol), "gemm_cfg_row")
        rows.append(tuple(buf))
    return cols, rows


_menu_cache: List[Tuple[int, ...]] = []
_cols_cache: List[str] = []


def menu_row(cfg_id: int) -> Tuple[int, ...]:
    """Knob tuple of one menu entry (the menu is read once)."""
    if not _menu_cache:
        _menu_cache.extend(menu()[1])
    return _menu_cache[cfg_id]


def menu_columns() -> List[str]:
    if not _cols_cache:
        _cols_cache.extend(lib.gemm_cfg_col_name(i).decode() for i in range(lib.gemm_cfg_num_cols()))
    return list(_cols_cache)


def cfg_find(knobs) -> int:
    ncol = lib.gemm_cfg_num_cols()
    k = list(knobs)
    if len(k) != ncol:
        return -1
    arr = (ctypes.c_int * ncol)(*[int(v) for v in k])
    return int(lib.gemm_cfg_find(arr, ncol))
