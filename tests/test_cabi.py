"""The C-ABI library loads, exports every function include/*.h declares, and
rejects bad arguments on the host.  CPU only: no call here reaches a device."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from attention_decode import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = []
    for header in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names += re.findall(r"ADB_API\s+[\w\s\*]+?\b(adb_\w+)\s*\(", text)
    return sorted(set(names))


def test_headers_declare_the_entry_points():
    names = declared_functions()
    for expected in ("adb_decode", "adb_decode_partial", "adb_combine", "adb_decode_workspace_size"):
        assert expected in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load_library()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.PROTOTYPES, f"{name} has no ctypes prototype"


def test_version_and_empty_last_error():
    lib = _lib.load_library()
    assert b"sm_100a" in lib.adb_version()
    assert isinstance(lib.adb_last_error(), bytes)


@pytest.mark.parametrize(
    "shape,status,pattern",
    [
        ((0, 32, 8, 129, 64), _lib.ADB_ERR_INVALID_ARGUMENT, "positive"),
        ((1, 32, 0, 129, 64), _lib.ADB_ERR_INVALID_ARGUMENT, "positive"),
        ((1, 32, 8, 0, 64), _lib.ADB_ERR_INVALID_ARGUMENT, "positive"),
        ((1, 31, 8, 129, 64), _lib.ADB_ERR_INVALID_ARGUMENT, "divisible"),
        ((1, 32, 16, 129, 64), _lib.ADB_ERR_UNSUPPORTED, "group"),
        ((1, 32, 4, 129, 64) , _lib.ADB_OK, None),
        ((1, 32, 8, 129, 96), _lib.ADB_ERR_UNSUPPORTED, "head dimension"),
        ((1, 32, 8, 129, 32), _lib.ADB_ERR_UNSUPPORTED, "head dimension"),
        ((1, 32, 8, 2**31, 64), _lib.ADB_ERR_INVALID_ARGUMENT, "kv_len"),
    ],
)
def test_workspace_query_validates_shapes_on_host(shape, status, pattern):
    if status == _lib.ADB_OK:
        pytest.skip("valid shape: the query would touch the device")
    lib = _lib.load_library()
    out = ctypes.c_size_t(0)
    rc = lib.adb_decode_workspace_size(*shape, 0, 0, ctypes.byref(out), None)
    assert rc == status
    assert re.search(pattern, _lib.last_error(lib))


def test_null_pointers_are_rejected_before_launch():
    lib = _lib.load_library()
    rc = lib.adb_decode(None, None, None, None, None, 1, 32, 8, 129, 64, None, 0, 0, 0, None)
    assert rc == _lib.ADB_ERR_INVALID_ARGUMENT
    assert "non-null" in _lib.last_error(lib)
    rc = lib.adb_combine(None, 0, None, 0, 1, 1, 64, None, 0, None)
    assert rc == _lib.ADB_ERR_INVALID_ARGUMENT


def test_check_raises_typed_error():
    lib = _lib.load_library()
    lib.adb_combine(None, 0, None, 0, 1, 1, 64, None, 0, None)
    with pytest.raises(_lib.AttentionDecodeError) as info:
        _lib.check(lib, _lib.ADB_ERR_INVALID_ARGUMENT)
    assert isinstance(info.value, RuntimeError)
    assert info.value.status == _lib.ADB_ERR_INVALID_ARGUMENT


def test_python_api_rejects_cpu_inputs():
    """tests/test_attention_decode.py:242-251."""
    import torch

    from attention_decode import attention_decode

    q = torch.randn(1, 32, 1, 64, dtype=torch.bfloat16)
    k = torch.randn(1, 8, 129, 64, dtype=torch.bfloat16)
    with pytest.raises((ValueError, RuntimeError, TypeError), match="(?i)cuda|device"):
        attention_decode(q, k, k)
    with pytest.raises(TypeError):
        attention_decode(None, k, k)


def test_exchange_arguments_are_checked_on_host():
    lib = _lib.load_library()
    size = ctypes.c_size_t(0)
    assert lib.adb_exchange_size(64, 128, 9, ctypes.byref(size)) == _lib.ADB_ERR_UNSUPPORTED
    assert lib.adb_exchange_size(64, 96, 2, ctypes.byref(size)) == _lib.ADB_ERR_UNSUPPORTED
    assert lib.adb_exchange_size(0, 128, 2, ctypes.byref(size)) == _lib.ADB_ERR_INVALID_ARGUMENT
    assert lib.adb_exchange_size(64, 128, 8, ctypes.byref(size)) == _lib.ADB_OK
    # 256-byte header, then two parities of 8 ranks' [64, 128] acc and [64, 2] (m, l)
    assert size.value == 256 + 2 * 8 * 64 * 128 * 4 + 2 * 8 * 64 * 2 * 4
    rc = lib.adb_decode_exchange(None, None, None, None, 1, 64, 8, 1024, 128, None, 2, 0, None, 0, 0, 0, None)
    assert rc == _lib.ADB_ERR_INVALID_ARGUMENT and "exchange" in _lib.last_error(lib)
    bases = (ctypes.c_void_p * 2)(256, 512)
    rc = lib.adb_decode_exchange(None, None, None, None, 1, 64, 8, 1024, 128, bases, 2, 2, None, 0, 0, 0, None)
    assert rc == _lib.ADB_ERR_INVALID_ARGUMENT and "rank" in _lib.last_error(lib)
    rc = lib.adb_exchange_merge(None, 2, 64, 128, None, 1000, 0, None)
    assert rc == _lib.ADB_ERR_INVALID_ARGUMENT
    rc = lib.adb_exchange_merge(256, 2, 64, 128, 512, 0, 0, None)
    assert rc == _lib.ADB_ERR_INVALID_ARGUMENT and "timeout" in _lib.last_error(lib)


def test_paged_arguments_are_checked_on_host():
    lib = _lib.load_library()
    args = lambda page, layout, table=1: (  # noqa: E731
        None, None, None, table, 4, 1, None, 2, 32, 8, 128, 16, page, 4, layout, None, 0, 0, 0, None)
    assert lib.adb_decode_paged(*args(16, 0, table=None)) == _lib.ADB_ERR_INVALID_ARGUMENT
    assert lib.adb_decode_paged(*args(16, 7)) == _lib.ADB_ERR_INVALID_ARGUMENT
    assert "layout" in _lib.last_error(lib)
    for page in (12, 4, 0, 3 << 20):
        assert lib.adb_decode_paged(*args(page, 0)) == _lib.ADB_ERR_UNSUPPORTED
        assert "power of two" in _lib.last_error(lib)


def test_append_arguments_are_checked_on_host():
    lib = _lib.load_library()
    rc = lib.adb_decode_append(None, None, None, None, None, None, None, 1, 32, 8, 128, 128, None, 0, 0, 0, None)
    assert rc == _lib.ADB_ERR_INVALID_ARGUMENT and "append" in _lib.last_error(lib)


def test_extension_object_has_the_reference_method_and_the_additions():
    """attention_decode/__init__.py:8-23 binds `forward`; the additions keep it."""
    import attention_decode
    from attention_decode import sharded

    ext = attention_decode._get_extension()
    # a pybind function: its signature is the first line of its docstring
    assert ext.forward.__doc__.startswith("forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor")
    assert callable(ext.forward_partial) and callable(ext.combine)
    assert sharded.attention_decode_sharded is sharded.attention_decode_sequence_sharded


def test_header_and_library_serve_a_plain_c_host(tmp_path):
    """A C program compiled against include/*.h and linked to the library
    (what a cgo / JNI / C++ host does) gets the documented answers."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib = _lib.load_library()
    lib_dir = str(_lib.LIB_PATH.parent)
    exe = tmp_path / "c_abi_host"
    build = subprocess.run(
        [cc, "-std=c99", "-Wall", "-Werror", f"-I{ROOT / 'include'}", str(ROOT / "tests" / "c_abi_host.c"),
         f"-L{lib_dir}", "-l:" + _lib.LIB_NAME, f"-Wl,-rpath,{lib_dir}", "-o", str(exe)],
        capture_output=True, text=True,
    )
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "all host checks passed" in run.stdout
    del lib
