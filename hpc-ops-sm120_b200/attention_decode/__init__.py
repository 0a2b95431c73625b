"""BF16 split-K attention decode for NVIDIA B200 (sm_100a).

Drop-in for the reference package's entry point
``attention_decode(q, k, v)`` (attention_decode/__init__.py:26-39): same
argument meaning, tensor layouts and error behaviour, with two compatible
extensions -- an optional per-sequence ``seqlens`` and head groups of 8.

Q: [B, Hq, 1, D]; K, V: [B, Hkv, S, D]; all BF16, contiguous, on one CUDA
device.  D is 64 or 128 and Hq / Hkv is 1, 4 or 8.  Work is enqueued on the
current CUDA stream with no host synchronisation, so calls can be captured in
CUDA graphs.  The kernels live in libattention_decode_b200.so (C ABI,
include/attention_decode_b200.h); there is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
from functools import lru_cache

from . import _lib
from ._lib import AttentionDecodeError

__all__ = [
    "attention_decode",
    "attention_decode_append",
    "attention_decode_fp8",
    "attention_decode_paged",
    "attention_decode_partial",
    "combine_partials",
    "workspace_bytes",
    "read_error_flag",
    "AttentionDecodeError",
]

_GROUPS = (1, 4, 8)
_DIMS = (64, 128)
_ws_cache: dict = {}


def _torch():
    import torch

    return torch


def _fail(message: str):
    # The reference raises these from TORCH_CHECK (c10::Error -> RuntimeError),
    # csrc/decode.cu:225-244.
    raise RuntimeError(message)


def _validate(q, k, v, seqlens=None):
    """Mirror of the reference's checks (attention_decode/__init__.py:35-38
    and csrc/decode.cu:225-241), with the INT_MAX size limit dropped (64-bit
    indexing) and G = 8 accepted.  Written as straight-line checks: this runs
    on every decode call."""
    torch = _torch()
    Tensor = torch.Tensor
    if not (isinstance(q, Tensor) and isinstance(k, Tensor) and isinstance(v, Tensor)):
        raise TypeError("Q, K, and V must be tensors")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("Q, K, and V must be CUDA tensors")
    bf16 = torch.bfloat16
    if q.dtype is not bf16 or k.dtype is not bf16 or v.dtype is not bf16:
        _fail("Q/K/V dtype must be BF16 (bfloat16)")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        _fail("Q/K/V must have rank four")
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        _fail("Q/K/V must be contiguous")
    if q.requires_grad or k.requires_grad or v.requires_grad:
        _fail("attention_decode is forward inference only; no backward/grad support")
    if q.numel() == 0 or k.numel() == 0 or v.numel() == 0:
        _fail("empty tensors are unsupported")
    if q.device != k.device or q.device != v.device:
        _fail("Q/K/V device must match")
    qs, ks = q.shape, k.shape
    if ks != v.shape:
        _fail("K/V shape must match")
    if qs[2] != 1:
        _fail("query length must be 1")
    if qs[0] != ks[0] or qs[3] != ks[3]:
        _fail("Q/K/V batch and head dimension must match")
    if qs[1] % ks[1] != 0:
        _fail("query heads must be divisible by KV heads")
    if qs[1] // ks[1] not in _GROUPS:
        _fail("supported GQA group sizes are 1, 4 and 8")
    if qs[3] not in _DIMS:
        _fail("head dimension must be 64 or 128")
    if seqlens is not None:
        if not isinstance(seqlens, Tensor):
            raise TypeError("seqlens must be a tensor")
        if seqlens.device != q.device:
            _fail("seqlens must be on the same CUDA device as Q/K/V")
        if seqlens.dtype != torch.int32:
            _fail("seqlens dtype must be int32")
        if seqlens.dim() != 1 or seqlens.shape[0] != qs[0] or not seqlens.is_contiguous():
            _fail("seqlens must be a contiguous [batch] tensor")


def workspace_bytes(batch, q_heads, kv_heads, kv_len, head_dim, has_seqlens=False, device=0) -> tuple[int, int]:
    """(workspace bytes, scheduler-header bytes) one decode call needs
    (adb_decode_workspace_size)."""
    key = (batch, q_heads, kv_heads, kv_len, head_dim, bool(has_seqlens), device)
    cached = _ws_cache.get(key)
    if cached is not None:
        return cached
    lib = _lib.load_library()
    total, header = ctypes.c_size_t(0), ctypes.c_size_t(0)
    _lib.check(
        lib,
        lib.adb_decode_workspace_size(
            batch, q_heads, kv_heads, kv_len, head_dim, int(bool(has_seqlens)), device,
            ctypes.byref(total), ctypes.byref(header),
        ),
    )
    _ws_cache[key] = (total.value, header.value)
    return _ws_cache[key]


# One workspace per (device, stream): calls on one stream are ordered, and each
# completed call leaves its scheduler header (the first `header` bytes) zero
# again, so no per-call memset is needed while the header fits in the prefix
# known to be zero.  A call whose header is larger than that prefix (another
# problem shape wrote segment data there) lets the library zero it.
# Concurrent streams get separate workspaces.  (The reference allocates its
# partial buffer per call from the caching allocator, csrc/decode.cu:205.)
_stream_workspaces: dict = {}
_MAX_STREAM_WORKSPACES = 64


class _StreamWorkspace:
    __slots__ = ("buf", "clean")

    def __init__(self, buf):
        self.buf = buf
        self.clean = buf.numel()  # bytes known to be zero


def _workspace(device_obj, device: int, stream: int, nbytes: int, header: int):
    torch = _torch()
    nbytes = max(nbytes, 256)
    if torch._C._cuda_isCurrentStreamCapturing():
        # A captured call owns its buffer in the graph's pool; the library's
        # header memset is captured with it.
        return torch.empty(nbytes, dtype=torch.uint8, device=device_obj), 0
    key = (device, stream)
    ws = _stream_workspaces.get(key)
    if ws is None or ws.buf.numel() < nbytes:
        if ws is None and len(_stream_workspaces) >= _MAX_STREAM_WORKSPACES:
            # Buffers are freed stream-ordered on the stream that used them.
            _stream_workspaces.pop(next(iter(_stream_workspaces)))
        ws = _StreamWorkspace(torch.zeros(nbytes, dtype=torch.uint8, device=device_obj))
        _stream_workspaces[key] = ws
    flags = _lib.ADB_FLAG_HEADER_ZEROED if header <= ws.clean else 0
    ws.clean = header  # after the call only its own header is guaranteed zero
    return ws.buf, flags


def _launch(q, k, v, seqlens, out=None, acc=None, ml=None):
    torch = _torch()
    lib = _lib.load_library()
    batch, q_heads, _, head_dim = q.shape
    kv_heads, kv_len = k.shape[1], k.shape[2]
    device = q.device.index if q.device.index is not None else torch.cuda.current_device()
    nbytes, header = workspace_bytes(batch, q_heads, kv_heads, kv_len, head_dim, seqlens is not None, device)
    stream = torch._C._cuda_getCurrentRawStream(device)
    workspace, flags = _workspace(q.device, device, stream, nbytes, header)
    lens = seqlens.data_ptr() if seqlens is not None else None
    if out is not None:
        status = lib.adb_decode(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), lens, out.data_ptr(),
            batch, q_heads, kv_heads, kv_len, head_dim,
            workspace.data_ptr(), workspace.numel(), flags, device, stream,
        )
    else:
        status = lib.adb_decode_partial(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), lens, acc.data_ptr(), ml.data_ptr(),
            batch, q_heads, kv_heads, kv_len, head_dim,
            workspace.data_ptr(), workspace.numel(), flags, device, stream,
        )
    _lib.check(lib, status)


def _launch_exchange(q, k, v, seqlens, bases, rank: int, out=None, timeout_us: int = 0):
    """adb_decode_exchange: partial decode whose states go to slot `rank` of
    every exchange buffer in `bases` (device addresses as mapped here).  With
    `out`, adb_decode_exchange_merged: the same launch also waits for every
    rank's states and merges them into `out` (ranks on distinct GPUs only)."""
    torch = _torch()
    lib = _lib.load_library()
    batch, q_heads, _, head_dim = q.shape
    kv_heads, kv_len = k.shape[1], k.shape[2]
    device = q.device.index if q.device.index is not None else torch.cuda.current_device()
    nbytes, header = workspace_bytes(batch, q_heads, kv_heads, kv_len, head_dim, seqlens is not None, device)
    stream = torch._C._cuda_getCurrentRawStream(device)
    workspace, flags = _workspace(q.device, device, stream, nbytes, header)
    lens = seqlens.data_ptr() if seqlens is not None else None
    array = (ctypes.c_void_p * len(bases))(*bases)
    if out is not None:
        _lib.check(
            lib,
            lib.adb_decode_exchange_merged(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), lens, batch, q_heads, kv_heads, kv_len, head_dim,
                array, len(bases), rank, out.data_ptr(), timeout_us, workspace.data_ptr(), workspace.numel(),
                flags, device, stream,
            ),
        )
        return
    _lib.check(
        lib,
        lib.adb_decode_exchange(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), lens, batch, q_heads, kv_heads, kv_len, head_dim,
            array, len(bases), rank, workspace.data_ptr(), workspace.numel(), flags, device, stream,
        ),
    )


def attention_decode(q, k, v, seqlens=None):
    """Forward-only single-query attention for contiguous BF16 CUDA tensors.

    Q: [B,Hq,1,D], K/V: [B,Hkv,S,D].  D is 64 or 128 and Hq/Hkv is 1, 4 or
    8.  ``seqlens`` (optional int32 [B] CUDA tensor) restricts sequence b to
    its first seqlens[b] tokens of the padded cache; a length of 0 gives a
    zero row.  Returns a new [B,Hq,1,D] BF16 tensor.  Uses the current CUDA
    stream.  The type and device checks are the reference's Python ones
    (attention_decode/__init__.py:35-38); the rest are done in C++ by the
    extension's ``forward`` with the reference's messages.
    """
    torch = _torch()
    Tensor = torch.Tensor
    if not (isinstance(q, Tensor) and isinstance(k, Tensor) and isinstance(v, Tensor)):
        raise TypeError("Q, K, and V must be tensors")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("Q, K, and V must be CUDA tensors")
    if seqlens is not None and not isinstance(seqlens, Tensor):
        raise TypeError("seqlens must be a tensor")
    return _get_extension().forward(q, k, v, seqlens)


def attention_decode_fp8(q, k, v, seqlens=None, *, k_scale=1.0, v_scale=1.0):
    """Decode over an FP8 (``torch.float8_e4m3fn``) K/V cache that stands for
    ``k * k_scale`` and ``v * v_scale`` (per-tensor scales).  Q is BF16
    [B,Hq,1,128]; K/V are [B,Hkv,S,128] e4m3.  Half the bytes of the BF16
    path; the reference reads BF16 only.  Returns BF16 [B,Hq,1,128].
    """
    torch = _torch()
    Tensor = torch.Tensor
    if not (isinstance(q, Tensor) and isinstance(k, Tensor) and isinstance(v, Tensor)):
        raise TypeError("Q, K, and V must be tensors")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("Q, K, and V must be CUDA tensors")
    if q.dtype is not torch.bfloat16:
        _fail("Q dtype must be BF16 (bfloat16)")
    if k.dtype is not torch.float8_e4m3fn or v.dtype is not torch.float8_e4m3fn:
        _fail("K/V dtype must be float8_e4m3fn")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        _fail("Q/K/V must have rank four")
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        _fail("Q/K/V must be contiguous")
    if q.device != k.device or q.device != v.device:
        _fail("Q/K/V device must match")
    if k.shape != v.shape:
        _fail("K/V shape must match")
    if q.shape[2] != 1:
        _fail("query length must be 1")
    if q.shape[0] != k.shape[0] or q.shape[3] != k.shape[3]:
        _fail("Q/K/V batch and head dimension must match")
    if q.shape[1] % k.shape[1] != 0:
        _fail("query heads must be divisible by KV heads")
    if seqlens is not None and (seqlens.dtype != torch.int32 or seqlens.dim() != 1
                                or seqlens.shape[0] != q.shape[0] or seqlens.device != q.device):
        _fail("seqlens must be an int32 [batch] tensor on Q's device")
    lib = _lib.load_library()
    batch, q_heads, _, head_dim = q.shape
    kv_heads, kv_len = k.shape[1], k.shape[2]
    device = q.device.index if q.device.index is not None else torch.cuda.current_device()
    nbytes, header = workspace_bytes(batch, q_heads, kv_heads, kv_len, head_dim, seqlens is not None, device)
    stream = torch._C._cuda_getCurrentRawStream(device)
    workspace, flags = _workspace(q.device, device, stream, nbytes, header)
    out = torch.empty_like(q)
    _lib.check(
        lib,
        lib.adb_decode_fp8(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), seqlens.data_ptr() if seqlens is not None else None,
            out.data_ptr(), batch, q_heads, kv_heads, kv_len, head_dim, float(k_scale), float(v_scale),
            workspace.data_ptr(), workspace.numel(), flags, device, stream,
        ),
    )
    return out


def attention_decode_append(q, k_new, v_new, k_cache, v_cache, seqlens):
    """One decode step with this step's token appended (fuses the cache
    append of a decode loop into the decode; the reference has no such step).

    ``k_cache``/``v_cache`` [B,Hkv,S_cap,D] hold ``seqlens[b]`` tokens of
    sequence b; ``k_new``/``v_new`` [B,Hkv,1,D] are the new token.  Returns
    attention over the cached tokens and the new one (BF16 [B,Hq,1,D]) and
    writes the new token into the caches at position ``seqlens[b]``.
    ``seqlens`` is not modified: add one to it after the call.  A full cache
    (``seqlens[b] >= S_cap``) is not written and sets bit 8 of
    :func:`read_error_flag`.
    """
    torch = _torch()
    if seqlens is None:
        raise TypeError("attention_decode_append needs seqlens")
    _validate(q, k_cache, v_cache, seqlens)
    for name, t in (("k_new", k_new), ("v_new", v_new)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a tensor")
        if not t.is_cuda or t.device != q.device:
            raise ValueError(f"{name} must be a CUDA tensor on Q's device")
        if t.dtype is not torch.bfloat16 or not t.is_contiguous():
            _fail(f"{name} must be a contiguous BF16 tensor")
        if tuple(t.shape) != (k_cache.shape[0], k_cache.shape[1], 1, k_cache.shape[3]):
            _fail(f"{name} must have shape [batch, kv_heads, 1, head_dim]")
    lib = _lib.load_library()
    batch, q_heads, _, head_dim = q.shape
    kv_heads, capacity = k_cache.shape[1], k_cache.shape[2]
    device = q.device.index if q.device.index is not None else torch.cuda.current_device()
    nbytes, header = workspace_bytes(batch, q_heads, kv_heads, capacity, head_dim, True, device)
    stream = torch._C._cuda_getCurrentRawStream(device)
    workspace, flags = _workspace(q.device, device, stream, nbytes, header)
    out = torch.empty_like(q)
    _lib.check(
        lib,
        lib.adb_decode_append(
            q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
            seqlens.data_ptr(), out.data_ptr(), batch, q_heads, kv_heads, capacity, head_dim,
            workspace.data_ptr(), workspace.numel(), flags, device, stream,
        ),
    )
    return out


_PAGED_LAYOUTS = {"HND": _lib.ADB_PAGED_HND, "NHD": _lib.ADB_PAGED_NHD}


def attention_decode_paged(q, k_cache, v_cache, block_table, seqlens, *, layout="HND"):
    """Decode over a paged KV cache (the layout of a serving engine's cache;
    the reference takes contiguous caches only).

    Q: [B,Hq,1,D] BF16.  ``k_cache``/``v_cache``: pools of pages, BF16,
    ``layout="HND"``: [num_blocks, Hkv, page_size, D] or ``"NHD"``:
    [num_blocks, page_size, Hkv, D]; page_size a power of two from 8.
    ``block_table``: int32 [B, max_blocks] (page j of sequence b is
    block_table[b, j]; rows may be padded with any value past a sequence's
    last page).  ``seqlens``: int32 [B], clamped to [0, max_blocks *
    page_size].  Returns a new [B,Hq,1,D] BF16 tensor.  Uses the current
    CUDA stream.
    """
    torch = _torch()
    if layout not in _PAGED_LAYOUTS:
        raise ValueError(f"layout must be 'HND' or 'NHD' (got {layout!r})")
    Tensor = torch.Tensor
    for name, t in (("Q", q), ("k_cache", k_cache), ("v_cache", v_cache), ("block_table", block_table), ("seqlens", seqlens)):
        if not isinstance(t, Tensor):
            raise TypeError(f"{name} must be a tensor")
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if t.device != q.device:
            _fail(f"{name} must be on Q's device")
    bf16 = torch.bfloat16
    if q.dtype is not bf16 or k_cache.dtype is not bf16 or v_cache.dtype is not bf16:
        _fail("Q/K/V dtype must be BF16 (bfloat16)")
    if q.dim() != 4 or k_cache.dim() != 4 or v_cache.dim() != 4:
        _fail("Q and the caches must have rank four")
    if not (q.is_contiguous() and k_cache.is_contiguous() and v_cache.is_contiguous()):
        _fail("Q/K/V must be contiguous")
    if k_cache.shape != v_cache.shape:
        _fail("K/V cache shapes must match")
    if q.shape[2] != 1:
        _fail("query length must be 1")
    if layout == "HND":
        num_blocks, kv_heads, page_size, head_dim = k_cache.shape
    else:
        num_blocks, page_size, kv_heads, head_dim = k_cache.shape
    batch, q_heads = q.shape[0], q.shape[1]
    if q.shape[3] != head_dim:
        _fail("Q/K/V batch and head dimension must match")
    if q_heads % kv_heads != 0:
        _fail("query heads must be divisible by KV heads")
    if q_heads // kv_heads not in _GROUPS:
        _fail("supported GQA group sizes are 1, 4 and 8")
    if head_dim not in _DIMS:
        _fail("head dimension must be 64 or 128")
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.shape[0] != batch or block_table.stride(1) != 1:
        _fail("block_table must be an int32 [batch, max_blocks] tensor with contiguous rows")
    if seqlens.dtype != torch.int32 or seqlens.dim() != 1 or seqlens.shape[0] != batch or not seqlens.is_contiguous():
        _fail("seqlens must be a contiguous int32 [batch] tensor")
    lib = _lib.load_library()
    device = q.device.index if q.device.index is not None else torch.cuda.current_device()
    max_blocks = block_table.shape[1]
    nbytes, header = workspace_bytes(batch, q_heads, kv_heads, max_blocks * page_size, head_dim, True, device)
    stream = torch._C._cuda_getCurrentRawStream(device)
    workspace, flags = _workspace(q.device, device, stream, nbytes, header)
    out = torch.empty_like(q)
    _lib.check(
        lib,
        lib.adb_decode_paged(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_table.data_ptr(), block_table.stride(0),
            seqlens.data_ptr(), out.data_ptr(), batch, q_heads, kv_heads, head_dim, num_blocks, page_size,
            max_blocks, _PAGED_LAYOUTS[layout], workspace.data_ptr(), workspace.numel(), flags, device, stream,
        ),
    )
    return out


def attention_decode_partial(q, k, v, seqlens=None, *, out_acc=None, out_ml=None):
    """Unnormalised decode state over this call's KV, for sequence sharding.

    Returns ``(acc, ml)``: acc FP32 [B, Hq, D] = sum_t exp(s_t - m) V_t and ml
    FP32 [B, Hq, 2] = (m, l) with m the max logit (natural units) and
    l = sum_t exp(s_t - m).  ``out_acc``/``out_ml`` may supply contiguous
    FP32 buffers of those shapes.  Merge states with :func:`combine_partials`.
    """
    torch = _torch()
    _validate(q, k, v, seqlens)
    batch, q_heads, _, head_dim = q.shape
    acc = out_acc if out_acc is not None else torch.empty((batch, q_heads, head_dim), dtype=torch.float32, device=q.device)
    ml = out_ml if out_ml is not None else torch.empty((batch, q_heads, 2), dtype=torch.float32, device=q.device)
    for buf, shape in ((acc, (batch, q_heads, head_dim)), (ml, (batch, q_heads, 2))):
        if tuple(buf.shape) != shape or buf.dtype != torch.float32 or not buf.is_contiguous() or buf.device != q.device:
            _fail(f"partial-state buffers must be contiguous float32 {shape} on {q.device}")
    _launch(q, k, v, seqlens, acc=acc, ml=ml)
    return acc, ml


def combine_partials(acc, ml, out=None):
    """Merge R partial states into a BF16 output.

    ``acc`` FP32 [R, rows, D] and ``ml`` FP32 [R, rows, 2], each with
    contiguous rows inside a part and any stride between parts (so views into
    an all-gathered buffer work).  Returns BF16 [rows, D] (or writes ``out``).
    """
    torch = _torch()
    lib = _lib.load_library()
    if acc.dtype != torch.float32 or ml.dtype != torch.float32:
        _fail("partial states must be float32")
    if not (acc.is_cuda and ml.is_cuda):
        raise ValueError("partial states must be CUDA tensors")
    parts, rows, head_dim = acc.shape
    if tuple(ml.shape) != (parts, rows, 2):
        _fail("ml must have shape [parts, rows, 2]")
    if acc.stride(1) != head_dim or acc.stride(2) != 1 or ml.stride(1) != 2 or ml.stride(2) != 1:
        _fail("partial states must have contiguous rows")
    if out is None:
        out = torch.empty((rows, head_dim), dtype=torch.bfloat16, device=acc.device)
    elif out.dtype != torch.bfloat16 or not out.is_contiguous() or out.numel() != rows * head_dim:
        _fail("out must be a contiguous bf16 buffer of rows * head_dim elements")
    device = acc.device.index if acc.device.index is not None else torch.cuda.current_device()
    stream = torch.cuda.current_stream(acc.device).cuda_stream
    _lib.check(
        lib,
        lib.adb_combine(
            acc.data_ptr(), acc.stride(0), ml.data_ptr(), ml.stride(0), parts, rows, head_dim,
            out.data_ptr(), device, stream,
        ),
    )
    return out


def read_error_flag(device=0, reset=True) -> int:
    """Sticky device error word (non-zero if a kernel's bounded wait expired)."""
    lib = _lib.load_library()
    flag = ctypes.c_int(0)
    _lib.check(lib, lib.adb_read_error_flag(device, ctypes.byref(flag), int(bool(reset))))
    return flag.value


@lru_cache(maxsize=1)
def _get_extension():
    """The PyTorch C++ extension (adb_torch_ext.so, built in-tree from
    csrc/torch_binding.cpp): ``forward(q, k, v, seqlens=None)``,
    ``forward_partial`` and ``combine``.  Replaces the reference's JIT-built
    module (attention_decode/__init__.py:8-23, csrc/binding.cpp:3-8); there
    is no fallback if it is missing."""
    _torch()
    _lib.load_library()
    try:
        from . import adb_torch_ext
    except ImportError as exc:
        raise ImportError(
            "attention_decode/adb_torch_ext.so is missing or does not load: build it with "
            "`python -c 'import __graft_entry__ as g; g.build()'` from the repository root"
        ) from exc
    return adb_torch_ext
