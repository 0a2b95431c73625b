"""FP8 (e4m3) K/V cache: the kernel's output against the CPU oracle over the
values the cache stands for (bytes decoded by the oracle times the
per-tensor scales), with the BF16 path's tolerance.  Padding past a
sequence's length holds the e4m3 NaN code and must not reach the output."""

from __future__ import annotations

import pytest
import torch

import attention_decode as ad
from helpers import SEED, check, inputs, oracle_reference_fp8

pytestmark = pytest.mark.gpu


def quantize(x):
    """Per-tensor e4m3 quantisation: (codes, scale) with amax mapped to 448."""
    scale = float(x.float().abs().max()) / 448.0
    return (x.float() / scale).to(torch.float8_e4m3fn), scale


@pytest.mark.parametrize("length", (1, 127, 128, 129, 1000, 4097))
@pytest.mark.parametrize("hq,hkv", ((32, 8), (32, 32), (64, 8)))
def test_fp8_matches_oracle(length, hq, hkv, device, record_property):
    q, k, v = inputs(device, length, 128, hkv, batch=2, hq=hq, seed=SEED + length)
    k8, ks = quantize(k)
    v8, vs = quantize(v * 3.0)
    out = ad.attention_decode_fp8(q, k8, v8, k_scale=ks, v_scale=vs)
    check(out, oracle_reference_fp8(q, k8, v8, ks, vs), q, record_property)


def test_fp8_sequence_lengths_and_nan_padding(device, record_property):
    lengths = [1, 0, 300, 4096, 2049, 64]
    q, k, v = inputs(device, 4096, 128, 8, batch=len(lengths), hq=64, seed=SEED + 7)
    k8, ks = quantize(k)
    v8, vs = quantize(v)
    nan = torch.tensor(0x7F, dtype=torch.uint8, device=device).view(torch.float8_e4m3fn)
    for b, n in enumerate(lengths):
        k8[b, :, n:] = nan
        v8[b, :, n:] = nan
    lens = torch.tensor(lengths, dtype=torch.int32, device=device)
    out = ad.attention_decode_fp8(q, k8, v8, lens, k_scale=ks, v_scale=vs)
    check(out, oracle_reference_fp8(q, k8, v8, ks, vs, lens), q, record_property)


def test_fp8_long_sequence_split_across_ctas(device, record_property):
    q, k, v = inputs(device, 65536 + 77, 128, 8, batch=1, hq=64, seed=SEED + 8)
    k8, ks = quantize(k)
    v8, vs = quantize(v)
    out = ad.attention_decode_fp8(q, k8, v8, k_scale=ks, v_scale=vs)
    check(out, oracle_reference_fp8(q, k8, v8, ks, vs), q, record_property)
    again = ad.attention_decode_fp8(q, k8, v8, k_scale=ks, v_scale=vs)
    check(again, out, q, None, atol=1e-3, rtol=2.0**-7)


def test_fp8_rejects_unsupported(device):
    q, k, v = inputs(device, 64, 64, 8, batch=1, hq=32, seed=1)
    k8, v8 = k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)
    with pytest.raises(RuntimeError, match="head dimension 128"):
        ad.attention_decode_fp8(q, k8, v8)
    q, k, v = inputs(device, 64, 128, 8, batch=1, hq=32, seed=1)
    with pytest.raises(RuntimeError, match="float8_e4m3fn"):
        ad.attention_decode_fp8(q, k, v)
    with pytest.raises(RuntimeError, match="scales"):
        ad.attention_decode_fp8(q, k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn), k_scale=0.0)
