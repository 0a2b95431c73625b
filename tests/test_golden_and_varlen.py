"""CUDA path against the reference's golden outputs, variable lengths
(including NaN padding that must not leak), and the partial/combine entry
points used by sequence sharding."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import attention_decode as ad
from golden.cases import CASES, GOLDEN_PATH
from helpers import check, from_bits, inputs, oracle_reference, to_bits
from oracle import attention_decode_oracle as oracle

pytestmark = pytest.mark.gpu
GOLDEN = np.load(GOLDEN_PATH)


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_golden_vectors(case, device, record_property):
    q, k, v, lens = case.inputs()
    tq, tk, tv = (from_bits(x, device) for x in (q, k, v))
    seqlens = torch.from_numpy(lens).to(device) if lens is not None else None
    out = ad.attention_decode(tq, tk, tv, seqlens)
    expected = from_bits(GOLDEN[f"{case.name}/out_bf16"], device)
    check(out, expected, tq, record_property)
    if case.name.startswith("single_token"):
        assert torch.equal(out, tv.repeat_interleave(case.q_heads // case.kv_heads, dim=1))


@pytest.mark.parametrize("lengths", [(1, 7, 8192, 3000), (0, 5, 64, 65), (129, 128, 127, 1), (8192, 8192, 8192, 8191)])
@pytest.mark.parametrize("dim,hq,hkv", ((128, 32, 8), (64, 64, 8), (128, 8, 8)))
def test_varlen_matches_per_sequence_oracle(lengths, dim, hq, hkv, device, record_property):
    batch, cap = len(lengths), 8192
    q, k, v = inputs(device, cap, dim, hkv, batch=batch, hq=hq, seed=77)
    seqlens = torch.tensor(lengths, dtype=torch.int32, device=device)
    # Padding past each length is NaN: it must never reach the output.
    for b, n in enumerate(lengths):
        k[b, :, n:] = float("nan")
        v[b, :, n:] = float("nan")
    out = ad.attention_decode(q, k, v, seqlens)
    expected = oracle_reference(q, k, v, seqlens)
    check(out, expected, q, record_property)
    for b, n in enumerate(lengths):
        if n == 0:
            assert not out[b].float().abs().sum().item()


# Two calls may merge their split segments in a different order (dynamic load
# balancing), so results agree to within one BF16 ulp rather than bit-exactly.
ULP = dict(atol=1e-3, rtol=2.0**-7)


def test_varlen_full_lengths_equal_uniform(device):
    q, k, v = inputs(device, 1000, 128, 8, batch=3, hq=32, seed=78)
    seqlens = torch.full((3,), 1000, dtype=torch.int32, device=device)
    a = ad.attention_decode(q, k, v, seqlens)
    b = ad.attention_decode(q, k, v)
    torch.testing.assert_close(a, b, **ULP)


def test_varlen_lengths_are_clamped(device):
    q, k, v = inputs(device, 300, 64, 8, batch=2, hq=32, seed=79)
    over = ad.attention_decode(q, k, v, torch.tensor([5000, -3], dtype=torch.int32, device=device))
    want = ad.attention_decode(q, k, v, torch.tensor([300, 0], dtype=torch.int32, device=device))
    torch.testing.assert_close(over, want, **ULP)
    assert not want[1].float().abs().sum().item()


@pytest.mark.parametrize("length,dim,hq,hkv,batch", ((4096, 128, 32, 8, 32), (131072, 128, 64, 8, 1), (777, 64, 8, 8, 5)))
def test_repeated_calls_agree(length, dim, hq, hkv, batch, device):
    """Load balancing changes how work is split between calls; every call must
    still be a correct decode (checked against the first within one ulp)."""
    q, k, v = inputs(device, length, dim, hkv, batch=batch, hq=hq, seed=83)
    first = ad.attention_decode(q, k, v)
    for _ in range(20):
        torch.testing.assert_close(ad.attention_decode(q, k, v), first, **ULP)


@pytest.mark.parametrize("length,dim,hq,hkv", ((4096, 128, 32, 8), (3001, 64, 64, 8), (1, 128, 8, 8)))
def test_partial_state_matches_oracle(length, dim, hq, hkv, device):
    q, k, v = inputs(device, length, dim, hkv, batch=2, hq=hq, seed=80)
    acc, ml = ad.attention_decode_partial(q, k, v)
    torch.cuda.synchronize(device)
    want_acc, want_m, want_l = oracle.partial_state(to_bits(q), to_bits(k), to_bits(v), 0, length)
    m = ml[..., 0].cpu().numpy()
    l = ml[..., 1].cpu().numpy()
    np.testing.assert_allclose(m, want_m, rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(l, want_l, rtol=1e-2, atol=1e-3)
    got = acc.cpu().numpy() / l[..., None]
    want = want_acc / want_l[..., None]
    np.testing.assert_allclose(got, want, atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("parts", (2, 3, 8))
@pytest.mark.parametrize("dim,hq,hkv", ((128, 64, 8), (64, 32, 8)))
def test_sequence_shards_merge_to_full_decode(parts, dim, hq, hkv, device, record_property):
    """Emulates sequence sharding on one GPU: each shard's partial state,
    stacked and merged by the combine entry point, equals the full decode."""
    length = 4096 + 37
    q, k, v = inputs(device, length, dim, hkv, batch=1, hq=hq, seed=81)
    bounds = [length * r // parts for r in range(parts + 1)]
    accs, mls = [], []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        acc, ml = ad.attention_decode_partial(q, k[:, :, lo:hi].contiguous(), v[:, :, lo:hi].contiguous())
        accs.append(acc.reshape(-1, dim))
        mls.append(ml.reshape(-1, 2))
    out = ad.combine_partials(torch.stack(accs), torch.stack(mls)).view_as(q)
    check(out, oracle_reference(q, k, v), q, record_property)


def test_combine_skips_empty_parts(device):
    q, k, v = inputs(device, 500, 128, 8, batch=1, hq=32, seed=82)
    acc, ml = ad.attention_decode_partial(q, k, v)
    empty_acc = torch.zeros_like(acc)
    empty_ml = torch.stack([torch.full_like(ml[..., 0], float("-inf")), torch.zeros_like(ml[..., 1])], -1)
    merged = ad.combine_partials(
        torch.stack([empty_acc.reshape(-1, 128), acc.reshape(-1, 128)]),
        torch.stack([empty_ml.reshape(-1, 2), ml.reshape(-1, 2)]),
    ).view_as(q)
    torch.testing.assert_close(merged, ad.attention_decode(q, k, v), atol=1e-2, rtol=1e-2)


def test_no_device_error_flag_after_tests(device):
    torch.cuda.synchronize(device)
    assert ad.read_error_flag(device.index or 0, reset=True) == 0


def test_extension_partial_and_combine_match_forward(device, record_property):
    """forward_partial on two token halves + combine == forward on all tokens."""
    q, k, v = inputs(device, 3001, 128, 8, batch=2, hq=32, seed=808)
    ext = ad._get_extension()
    full = ext.forward(q, k, v)
    halves = [ext.forward_partial(q, k[:, :, a:b].contiguous(), v[:, :, a:b].contiguous()) for a, b in ((0, 1500), (1500, 3001))]
    acc = torch.stack([h[0] for h in halves])
    ml = torch.stack([h[1] for h in halves])
    merged = ext.combine(acc, ml)
    check(merged, full, q, record_property, atol=1e-2, rtol=2.0**-7)
