"""The allocation-free entry point adb_decode_no_alloc, called through the C ABI.

Some callers of this library cannot allocate device memory themselves: a host
that binds the C ABI from another language while its device memory belongs
to a different allocator, or a serving loop that must not enter
cudaMalloc/cudaFree because they synchronise the device.  adb_decode_no_alloc
serves them with a fixed scratch array inside the library.  Here it must
give the same results as the regular entry point (adb_decode, reached through
attention_decode) and as the CPU oracle, within the tolerance of the other
parity tests, on two calls in a row (the second call finds the previous call's leftovers in the
shared array), and refuse a problem whose scratch does not fit.

This file sorts last so a stopping run has run every other test before it; it
also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from attention_decode import _lib, attention_decode
from helpers import ATOL, RTOL, check, inputs, oracle_reference

pytestmark = pytest.mark.gpu


def _no_alloc(lib, q, k, v, seqlens, out):
    batch, q_heads, _, head_dim = q.shape
    kv_heads, kv_len = k.shape[1], k.shape[2]
    device = q.device.index if q.device.index is not None else torch.cuda.current_device()
    return lib.adb_decode_no_alloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(),
        seqlens.data_ptr() if seqlens is not None else None, out.data_ptr(),
        batch, q_heads, kv_heads, kv_len, head_dim, device,
        torch.cuda.current_stream(q.device).cuda_stream,
    )


CASES = [
    # batch, q_heads, kv_heads, kv_len, head_dim, seqlens
    (32, 32, 8, 4096, 128, None),
    (3, 64, 8, 1000, 64, (1000, 1, 517)),
    (1, 8, 8, 1024, 128, None),
    (4, 32, 32, 129, 64, None),
]


@pytest.mark.parametrize("batch,hq,hkv,length,dim,lens", CASES)
def test_no_alloc_matches_regular_entry_point(batch, hq, hkv, length, dim, lens, cuda_device):
    lib = _lib.load_library()
    q, k, v = inputs(cuda_device, length, dim, hkv, batch=batch, hq=hq, seed=4242)
    seqlens = torch.tensor(lens, dtype=torch.int32, device=cuda_device) if lens is not None else None
    expected = attention_decode(q, k, v, seqlens)
    want = oracle_reference(q, k, v, seqlens)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _lib.check(lib, _no_alloc(lib, q, k, v, seqlens, out))
        torch.cuda.synchronize(cuda_device)
        assert torch.isfinite(out).all().item()
        torch.testing.assert_close(out, expected, atol=ATOL, rtol=RTOL)
        check(out, want, q)


def test_no_alloc_rejects_problems_larger_than_its_workspace(cuda_device):
    lib = _lib.load_library()
    q, k, v = inputs(cuda_device, 16, 128, 8, batch=1, hq=64, seed=1)
    out = torch.empty_like(q)
    # The shape arguments describe a problem whose scratch cannot fit in the
    # fixed array; the call must fail on the host before touching the device
    # buffers (which are far smaller than the shape claims).
    status = lib.adb_decode_no_alloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), None, out.data_ptr(),
        100000, 64, 8, 16, 128, cuda_device.index or 0,
        torch.cuda.current_stream(cuda_device).cuda_stream,
    )
    assert status == _lib.ADB_ERR_WORKSPACE
    message = _lib.last_error(lib)
    assert "fixed workspace" in message and str(8 << 20) in message
