"""ctypes binding of libattention_decode_b200.so (the C ABI in
include/attention_decode_b200.h).

This is the reference-side stub a maintainer would add in place of the
reference's JIT-built pybind extension (attention_decode/__init__.py:8-23,
csrc/binding.cpp:1-8): it loads the prebuilt in-tree shared library and
declares each entry point's argument types.  There is no fallback: if the
library is missing the import fails with instructions to build it.
"""

from __future__ import annotations

import ctypes
import os
from functools import lru_cache
from pathlib import Path

LIB_NAME = "libattention_decode_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

ADB_OK = 0
ADB_ERR_INVALID_ARGUMENT = 1
ADB_ERR_UNSUPPORTED = 2
ADB_ERR_DEVICE = 3
ADB_ERR_WORKSPACE = 4
ADB_ERR_CUDA = 5
ADB_FLAG_HEADER_ZEROED = 1
ADB_IPC_HANDLE_BYTES = 64
ADB_PAGED_HND = 0
ADB_PAGED_NHD = 1
ADB_ERROR_FLAG_PEER_TIMEOUT = 4
ADB_ERROR_FLAG_APPEND_FULL = 8

STATUS_NAMES = {
    ADB_OK: "ok",
    ADB_ERR_INVALID_ARGUMENT: "invalid argument",
    ADB_ERR_UNSUPPORTED: "unsupported",
    ADB_ERR_DEVICE: "unsupported device",
    ADB_ERR_WORKSPACE: "workspace",
    ADB_ERR_CUDA: "CUDA error",
}

# name -> (restype, argtypes); mirrors include/attention_decode_b200.h
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_int = ctypes.c_int
_size = ctypes.c_size_t
_uint = ctypes.c_uint
PROTOTYPES = {
    "adb_version": (ctypes.c_char_p, []),
    "adb_last_error": (ctypes.c_char_p, []),
    "adb_check_device": (_int, [_int]),
    "adb_decode_workspace_size": (
        _int,
        [_i64, _i64, _i64, _i64, _i64, _int, _int, ctypes.POINTER(_size), ctypes.POINTER(_size)],
    ),
    "adb_decode": (
        _int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _size, _uint, _int, _vp],
    ),
    "adb_decode_partial": (
        _int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _size, _uint, _int, _vp],
    ),
    "adb_decode_fp8": (
        _int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, ctypes.c_float,
         _vp, _size, _uint, _int, _vp],
    ),
    "adb_decode_append": (
        _int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _size, _uint, _int, _vp],
    ),
    "adb_decode_paged": (
        _int,
        [_vp, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int,
         _vp, _size, _uint, _int, _vp],
    ),
    "adb_decode_no_alloc": (
        _int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _int, _vp],
    ),
    "adb_combine": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _int, _vp]),
    "adb_exchange_size": (_int, [_i64, _i64, _int, ctypes.POINTER(ctypes.c_size_t)]),
    "adb_exchange_alloc": (_int, [ctypes.c_size_t, _int, ctypes.POINTER(_vp)]),
    "adb_exchange_free": (_int, [_vp, _int]),
    "adb_ipc_handle": (_int, [_vp, _int, ctypes.c_char_p]),
    "adb_ipc_open": (_int, [ctypes.c_char_p, _int, ctypes.POINTER(_vp)]),
    "adb_ipc_close": (_int, [_vp, _int]),
    "adb_decode_exchange": (
        _int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, ctypes.POINTER(_vp), _int, _int,
         _vp, ctypes.c_size_t, ctypes.c_uint, _int, _vp],
    ),
    "adb_exchange_merge": (_int, [_vp, _int, _i64, _i64, _vp, _i64, _int, _vp]),
    "adb_decode_exchange_merged": (
        _int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, ctypes.POINTER(_vp), _int, _int,
         _vp, _i64, _vp, ctypes.c_size_t, ctypes.c_uint, _int, _vp],
    ),
    "adb_read_error_flag": (_int, [_int, ctypes.POINTER(_int), _int]),
    "adb_launch_count": (_int, [ctypes.POINTER(_i64)]),
    "adb_timing_enable": (_int, [_int]),
    "adb_timing_read": (_int, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_i64)]),
}


class AttentionDecodeError(RuntimeError):
    """A failing C-ABI call; `status` is the adb_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


@lru_cache(maxsize=1)
def load_library(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load the shared library and declare every entry point's signature."""
    target = Path(path) if path is not None else LIB_PATH
    if not target.is_file():
        raise ImportError(
            f"{target} is missing: build it first with `python -c 'import __graft_entry__ as g; "
            f"g.build()'` from the repository root (no CPU fallback exists)"
        )
    lib = ctypes.CDLL(str(target))
    for name, (restype, argtypes) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def last_error(lib: ctypes.CDLL) -> str:
    raw = lib.adb_last_error()
    return raw.decode("utf-8", "replace") if raw else ""


def check(lib: ctypes.CDLL, status: int) -> None:
    """Raise AttentionDecodeError for a non-zero adb_status."""
    if status != ADB_OK:
        raise AttentionDecodeError(status, last_error(lib) or STATUS_NAMES.get(status, str(status)))
