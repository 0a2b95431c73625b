"""Decode with this step's token appended (attention_decode_append): the
output must equal the CPU oracle over the cache with the token written at
position seqlens[b] and one more token per sequence, the caches must hold the
new rows there afterwards and be unchanged everywhere else, and a full cache
must be reported (device error word) instead of written past its end."""

from __future__ import annotations

import pytest
import torch

import attention_decode as ad
from attention_decode import _lib
from helpers import check, inputs, oracle_reference

pytestmark = pytest.mark.gpu


def _case(device, lengths, capacity, dim, hq, hkv, seed):
    batch = len(lengths)
    q, k, v = inputs(device, capacity, dim, hkv, batch=batch, hq=hq, seed=seed)
    k_new, v_new = (x[:, :, :1].clone() for x in inputs(device, 1, dim, hkv, batch=batch, hq=hq, seed=seed + 1)[1:])
    lens = torch.tensor(lengths, dtype=torch.int32, device=device)
    return q, k, v, k_new, v_new, lens


def _expected_cache(k, v, k_new, v_new, lengths):
    k2, v2 = k.clone(), v.clone()
    for b, n in enumerate(lengths):
        if n < k.shape[2]:
            k2[b, :, n] = k_new[b, :, 0]
            v2[b, :, n] = v_new[b, :, 0]
    return k2, v2


@pytest.mark.parametrize("dim,hq,hkv", ((128, 32, 8), (64, 32, 32), (128, 64, 8), (64, 16, 4)))
def test_append_matches_oracle_and_writes_the_cache(dim, hq, hkv, device, record_property):
    capacity = 1100
    lengths = [0, 1, 63, 64, 127, 128, 129, capacity - 1, 700]
    q, k, v, k_new, v_new, lens = _case(device, lengths, capacity, dim, hq, hkv, seed=dim + hq)
    k2, v2 = _expected_cache(k, v, k_new, v_new, lengths)
    ad.read_error_flag(device.index or 0)
    out = ad.attention_decode_append(q, k_new, v_new, k, v, lens)
    torch.cuda.synchronize(device)
    assert torch.equal(k, k2) and torch.equal(v, v2), "cache rows other than the appended ones changed"
    check(out, oracle_reference(q, k2, v2, lens + 1), q, record_property)
    check(out, ad.attention_decode(q, k2, v2, lens + 1), q, None, atol=1e-2, rtol=2.0**-7)
    assert torch.equal(out[0], v_new[0].repeat_interleave(hq // hkv, dim=0)), "one-token row must be V exactly"
    assert ad.read_error_flag(device.index or 0) == 0


def test_append_long_sequences_split_across_ctas(device, record_property):
    lengths = [30000, 5, 65536 - 1, 12345]
    q, k, v, k_new, v_new, lens = _case(device, lengths, 65536, 128, 64, 8, seed=5)
    k2, v2 = _expected_cache(k, v, k_new, v_new, lengths)
    out = ad.attention_decode_append(q, k_new, v_new, k, v, lens)
    torch.cuda.synchronize(device)
    assert torch.equal(k, k2) and torch.equal(v, v2)
    check(out, oracle_reference(q, k2, v2, lens + 1), q, record_property)


def test_append_to_a_full_cache_is_reported(device):
    capacity = 256
    q, k, v, k_new, v_new, lens = _case(device, [capacity, 10], capacity, 128, 32, 8, seed=9)
    k_before, v_before = k.clone(), v.clone()
    ad.read_error_flag(device.index or 0)
    out = ad.attention_decode_append(q, k_new, v_new, k, v, lens)
    torch.cuda.synchronize(device)
    assert ad.read_error_flag(device.index or 0) & _lib.ADB_ERROR_FLAG_APPEND_FULL
    assert torch.equal(k[0], k_before[0]) and torch.equal(v[0], v_before[0])
    # the full sequence attends to its capacity plus the new token
    k_ext = torch.cat([k_before[:1], k_new[:1]], dim=2)
    v_ext = torch.cat([v_before[:1], v_new[:1]], dim=2)
    check(out[:1], oracle_reference(q[:1], k_ext, v_ext), q[:1])


def test_append_with_unaligned_cache(device, record_property):
    lengths = [300, 0, 1023]
    q, k, v, k_new, v_new, lens = _case(device, lengths, 1024, 128, 32, 8, seed=13)
    shifted = []
    for t in (k, v):
        storage = torch.empty(t.numel() + 1, dtype=t.dtype, device=device)
        view = storage[1:].view_as(t)
        view.copy_(t)
        shifted.append(view)
    ks, vs = shifted
    k2, v2 = _expected_cache(k, v, k_new, v_new, lengths)
    out = ad.attention_decode_append(q, k_new, v_new, ks, vs, lens)
    torch.cuda.synchronize(device)
    assert torch.equal(ks, k2) and torch.equal(vs, v2)
    check(out, oracle_reference(q, k2, v2, lens + 1), q, record_property)


def test_append_is_one_step_of_a_decode_loop(device, record_property):
    """Three steps: append + raise seqlens on the stream, as a serving loop does."""
    lengths = [5, 130, 0]
    q, k, v, _, _, lens = _case(device, lengths, 512, 128, 32, 8, seed=21)
    ref_k, ref_v = k.clone(), v.clone()
    ref_lens = lens.clone()
    for step in range(3):
        k_new, v_new = (x[:, :, :1].clone() for x in inputs(device, 1, 128, 8, batch=3, hq=32, seed=100 + step)[1:])
        out = ad.attention_decode_append(q, k_new, v_new, k, v, lens)
        lens += 1
        ref_k, ref_v = _expected_cache(ref_k, ref_v, k_new, v_new, ref_lens.tolist())
        ref_lens += 1
        check(out, oracle_reference(q, ref_k, ref_v, ref_lens), q, record_property, f"step{step}")
    assert torch.equal(k, ref_k) and torch.equal(v, ref_v)
