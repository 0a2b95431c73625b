"""Pins the CPU oracle (oracle/attention_decode_oracle.py) against golden
outputs of the reference's own FP32 oracle, and against the reference's
analytic known-answer tests.  CPU only."""

from __future__ import annotations

import math

import numpy as np
import pytest

from golden.cases import CASES, GOLDEN_PATH
from oracle import attention_decode_oracle as oracle

GOLDEN = np.load(GOLDEN_PATH)


def _run(case):
    q, k, v, lens = case.inputs()
    if lens is None:
        return oracle.reference_fp32(q, k, v)
    return oracle.reference_varlen_fp32(q, k, v, lens)


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_inputs_match_golden_checksum(case):
    assert bytes(GOLDEN[f"{case.name}/checksum"]).hex() == case.checksum()


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_matches_reference_golden(case):
    out32 = _run(case)
    want32 = GOLDEN[f"{case.name}/out_fp32"]
    want16 = GOLDEN[f"{case.name}/out_bf16"]
    assert out32.shape == want32.shape
    assert np.isfinite(out32).all()
    # FP32 agreement up to summation order (BLAS vs torch): 1e-5 relative.
    np.testing.assert_allclose(out32, want32, rtol=1e-5, atol=1e-5)
    # BF16-rounded outputs: identical except values whose FP32 result sits on a
    # rounding boundary, which may flip by one ulp under the FP32 noise.
    got16 = oracle.f32_to_bf16_bits(out32)
    differing = np.count_nonzero(got16 != want16)
    assert differing <= max(4, got16.size // 100)
    got, want = oracle.bf16_bits_to_f32(got16), oracle.bf16_bits_to_f32(want16)
    assert np.all(np.abs(got - want) <= np.maximum(1e-5, np.abs(want) * 2.0**-7))


def test_bf16_rounding_matches_torch():
    import torch

    rng = np.random.default_rng(7)
    x = np.concatenate(
        [rng.standard_normal(10000, dtype=np.float32) * 100, np.array([0.0, -0.0, np.inf, -np.inf], np.float32)]
    )
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(oracle.f32_to_bf16_bits(x), want)
    np.testing.assert_array_equal(oracle.bf16_bits_to_f32(want), torch.from_numpy(want.view(np.int16)).view(torch.bfloat16).float().numpy())


def test_oracle_matches_explicit_gqa_formula():
    """tests/test_attention_decode.py:228-239, on the numpy oracle."""
    q, k, v, _ = next(c for c in CASES if c.name == "gqa_formula").inputs()
    qf, kf, vf = (oracle.bf16_bits_to_f32(x) for x in (q, k, v))
    heads = []
    for head in range(32):
        kv_head = head // 4
        scores = qf[:, head] @ kf[:, kv_head].transpose(0, 2, 1)
        scores = scores / np.float32(math.sqrt(64))
        w = np.exp(scores - scores.max(-1, keepdims=True))
        w = w / w.sum(-1, keepdims=True)
        heads.append(w @ vf[:, kv_head])
    expected = oracle.f32_to_bf16_bits(np.stack(heads, axis=1).astype(np.float32))
    actual = oracle.reference(q, k, v)
    diff = np.abs(actual.astype(np.int32) - expected.astype(np.int32))
    assert diff.max() <= 1


def test_single_token_is_exact_value():
    """T=1 returns the mapped V exactly (tests/test_attention_decode.py:156-165)."""
    for name in ("single_token_d64", "single_token_d128_mha"):
        case = next(c for c in CASES if c.name == name)
        q, k, v, _ = case.inputs()
        group = case.q_heads // case.kv_heads
        expected = np.repeat(v, group, axis=1)
        np.testing.assert_array_equal(oracle.reference(q, k, v), expected)


def test_common_offset_is_uniform_mean():
    case = next(c for c in CASES if c.name == "common_offset")
    q, k, v, _ = case.inputs()
    mean = oracle.bf16_bits_to_f32(v).mean(axis=2, keepdims=True)
    expected = np.repeat(mean, 4, axis=1)
    np.testing.assert_allclose(oracle.reference_fp32(q, k, v), expected, atol=1e-5)


def test_gqa_grouping_distinguishes_floor_division():
    case = next(c for c in CASES if c.name == "gqa_grouping")
    q, k, v, _ = case.inputs()
    out = oracle.bf16_bits_to_f32(oracle.reference(q, k, v))
    for b in range(4):
        for hq in range(32):
            assert out[b, hq, 0, 0] == b * 8 + hq // 4


def test_separated_maxima_matches_constant_values():
    case = next(c for c in CASES if c.name == "separated_maxima")
    q, k, v, _ = case.inputs()
    out = oracle.bf16_bits_to_f32(oracle.reference(q, k, v))
    for hq in range(32):
        assert out[0, hq, 0, 0] == (hq // 4) / 8 + 0.125


@pytest.mark.parametrize("cuts", [(0, 100, 300), (0, 1, 299, 300), (0, 150, 150, 300)])
def test_partial_states_merge_to_full_result(cuts):
    """Split-K identity: merging per-range states equals the full softmax."""
    case = next(c for c in CASES if c.name == "varlen")
    q, k, v, _ = case.inputs()
    parts = [oracle.partial_state(q, k, v, lo, hi) for lo, hi in zip(cuts[:-1], cuts[1:])]
    merged = oracle.merge_states(*zip(*parts))
    full = oracle.reference_fp32(q, k, v).reshape(merged.shape)
    np.testing.assert_allclose(merged, full, rtol=2e-5, atol=2e-6)


def test_merge_of_only_empty_parts_is_zero():
    acc = np.zeros((3, 2, 64), np.float32)
    m = np.full((3, 2), -np.inf, np.float32)
    l = np.zeros((3, 2), np.float32)
    assert not np.any(oracle.merge_states(acc, m, l))


def test_varlen_zero_length_gives_zeros():
    case = next(c for c in CASES if c.name == "varlen")
    q, k, v, _ = case.inputs()
    out = oracle.reference_varlen_fp32(q, k, v, [0, 5, 300, 301])
    assert not np.any(out[0])
    np.testing.assert_allclose(out[3], oracle.reference_fp32(q[3:4], k[3:4], v[3:4])[0], rtol=1e-6, atol=1e-6)


def test_e4m3_decoding_matches_torch():
    """Pins the oracle's FP8 e4m3 decoder to torch's conversion on all 256 codes."""
    import torch

    codes = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    got = oracle.e4m3_to_f32(codes)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan], want[~nan])


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_torch_restatement_matches_reference_golden(case):
    """Pins oracle/reference_torch.py (the CPU baseline the benchmark times)
    against the same golden outputs of the reference's reference.py."""
    import torch

    from oracle import reference_torch

    q, k, v, lens = case.inputs()
    tq, tk, tv = (torch.from_numpy(x.view(np.int16)).view(torch.bfloat16) for x in (q, k, v))
    if lens is None:
        out32 = reference_torch.reference_fp32(tq, tk, tv).numpy()
    else:
        out32 = reference_torch.reference_varlen_fp32(tq, tk, tv, lens).numpy()
    want32 = GOLDEN[f"{case.name}/out_fp32"]
    assert out32.shape == want32.shape
    np.testing.assert_allclose(out32, want32, rtol=1e-5, atol=1e-5)
