"""Helpers shared by the tests: torch <-> BF16-bit conversion, the oracle on
torch tensors, and the tolerance check.

Tolerances: the reference contract is torch.testing.assert_close(atol=2e-2,
rtol=2e-2) against the BF16-rounded FP32 oracle (attention_decode/reference.py:11-12,
tests/test_attention_decode.py:60-78).  The north-star gate is stricter on
the relative term: atol=2e-2, rtol=1e-2, plus finiteness.  check() applies
the stricter one.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import attention_decode_oracle as oracle

ATOL = 2e-2
RTOL = 1e-2
SEED = 20261013  # tests/test_attention_decode.py:22


def to_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(bits: np.ndarray, device=None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
    return t.to(device) if device is not None else t


def oracle_reference(q, k, v, seqlens=None) -> torch.Tensor:
    """The CPU oracle on torch tensors; returns BF16 on q's device."""
    qb, kb, vb = to_bits(q), to_bits(k), to_bits(v)
    if seqlens is None:
        out = oracle.reference_fp32(qb, kb, vb)
    else:
        out = oracle.reference_varlen_fp32(qb, kb, vb, seqlens.cpu().numpy())
    return from_bits(oracle.f32_to_bf16_bits(out), q.device)


def oracle_reference_fp8(q, k8, v8, k_scale, v_scale, seqlens=None) -> torch.Tensor:
    """The CPU oracle over the values an e4m3 cache stands for (bytes decoded
    by the oracle, times the per-tensor scales); BF16 on q's device."""
    qb = to_bits(q)
    kf = oracle.e4m3_to_f32(k8.detach().contiguous().cpu().view(torch.uint8).numpy()) * np.float32(k_scale)
    vf = oracle.e4m3_to_f32(v8.detach().contiguous().cpu().view(torch.uint8).numpy()) * np.float32(v_scale)
    if seqlens is None:
        out = oracle.reference_fp32(qb, kf, vf)
    else:
        out = oracle.reference_varlen_fp32(qb, kf, vf, seqlens.cpu().numpy())
    return from_bits(oracle.f32_to_bf16_bits(out), q.device)


def inputs(device, length, dim=128, hkv=8, batch=1, seed=SEED, hq=32):
    """Seeded inputs generated on `device` (tests/test_extreme_decode.py:22-25)."""
    generator = torch.Generator(device=device).manual_seed(seed)
    return tuple(
        torch.randn(shape, generator=generator, device=device, dtype=torch.bfloat16)
        for shape in ((batch, hq, 1, dim), (batch, hkv, length, dim), (batch, hkv, length, dim))
    )


def check(output, expected, q=None, record_property=None, label="result", atol=ATOL, rtol=RTOL):
    if q is not None:
        assert output.shape == q.shape
        assert output.device == q.device
    assert output.dtype == torch.bfloat16
    assert torch.isfinite(output).all().item(), "output contains NaN or Inf"
    assert torch.isfinite(expected).all().item(), "reference contains NaN or Inf"
    absolute = (output.float() - expected.float()).abs()
    relative = absolute / expected.float().abs().clamp_min(1e-6)
    if record_property is not None:
        record_property(f"{label}_max_abs_error", absolute.max().item())
        record_property(f"{label}_max_rel_error", relative.max().item())
        record_property("atol", atol)
        record_property("rtol", rtol)
    torch.testing.assert_close(output, expected, atol=atol, rtol=rtol)
