"""CPU oracle for BF16 single-query attention decode -- TEST INFRASTRUCTURE.

This module is the checker, never the product: only tests/, the smoke test in
__graft_entry__.py and bench.py's CPU-baseline / reference arm may import it.
The product path (hpc-ops-sm120_b200/attention_decode) never calls it and has
no CPU fallback.

It restates, in numpy, the reference's FP32 oracle
``attention_decode.reference.reference_fp32`` (attention_decode/reference.py:47-60):

    grouped_q = q.float().reshape(B, Hkv, G, D)            # :55
    logits    = grouped_q @ k.float().transpose(-1, -2)    # :56
    logits   *= 1 / sqrt(D)                                # :57
    probs     = softmax(logits, dim=-1) in FP32            # :58
    out       = probs @ v.float()                          # :59
    return out.reshape(B, Hq, 1, D)                        # :60

and ``reference`` (reference.py:63-66), which rounds that to BF16.  BF16
tensors are carried as uint16 bit patterns (numpy has no bfloat16); rounding
FP32 -> BF16 is round-to-nearest-even, as torch's ``.to(torch.bfloat16)``.

Pinning: tests/test_oracle_golden.py checks this restatement against golden
outputs that tests/golden/make_golden.py produced by running the reference's
own reference.py on the same inputs (tests/golden/golden_vectors.npz).

Additions beyond the reference (same arithmetic, used to check the
extensions): per-sequence lengths (the reference has no varlen; each sequence
is the reference computation on its first L_b tokens) and the partial
(acc, m, l) state / merge used by split-K and sequence sharding, following
the reference's split partial and merge_splits (csrc/decode.cu:127-129,160,
169-184).
"""

from __future__ import annotations

import math

import numpy as np

ATOL = 2e-2  # reference.py:11
RTOL = 2e-2  # reference.py:12


# ---------------------------------------------------------------- bf16 bits
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact widening of BF16 bit patterns (uint16) to float32."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to BF16 (round to nearest, ties to even); NaN stays NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    rounded = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint16)
    rounded = np.where(np.isnan(x), np.uint16(0x7FC0), rounded)
    return rounded.astype(np.uint16)


def as_f32(x: np.ndarray) -> np.ndarray:
    """float32 view of an input given either as BF16 bits or as floats."""
    if x.dtype == np.uint16:
        return bf16_bits_to_f32(x)
    return np.ascontiguousarray(x, dtype=np.float32)


def e4m3_to_f32(bits: np.ndarray) -> np.ndarray:
    """Decode FP8 e4m3 bytes (OCP "fn" encoding: 1 sign, 4 exponent bits with
    bias 7, 3 mantissa bits, subnormals, no infinities, S.1111.111 is NaN) to
    float32, exactly.  Used to check the FP8 K/V extension (not in the
    reference, which reads BF16 only)."""
    b = np.ascontiguousarray(bits, dtype=np.uint8).astype(np.int32)
    sign = np.where(b & 0x80, -1.0, 1.0).astype(np.float32)
    exp = (b >> 3) & 0xF
    man = (b & 0x7).astype(np.float32)
    normal = (1.0 + man / 8.0) * np.exp2(exp.astype(np.float32) - 7.0)
    subnormal = (man / 8.0) * np.float32(2.0 ** -6)
    out = sign * np.where(exp == 0, subnormal, normal).astype(np.float32)
    return np.where((b & 0x7F) == 0x7F, np.float32(np.nan), out).astype(np.float32)


# ---------------------------------------------------------------- reference
def validate_shapes(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> tuple[int, int, int, int, int, int]:
    """Shape contract of reference.py:15-34 (dtype/device/layout do not apply)."""
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("Q, K, and V must be four-dimensional")
    if q.shape[2] != 1:
        raise ValueError("query sequence length must be 1")
    if k.shape != v.shape:
        raise ValueError("K and V shapes must match")
    if q.shape[0] != k.shape[0] or q.shape[3] != k.shape[3]:
        raise ValueError("Q and K/V batch size and head dimension must match")
    if min(q.shape) < 1 or min(k.shape) < 1:
        raise ValueError("all dimensions must be positive")
    if q.shape[1] % k.shape[1] != 0:
        raise ValueError("query head count must be divisible by KV head count")
    batch, query_heads, _, dim = q.shape
    kv_heads, length = k.shape[1], k.shape[2]
    return batch, query_heads, kv_heads, query_heads // kv_heads, length, dim


def _softmax_lastdim(logits: np.ndarray) -> np.ndarray:
    shifted = logits - logits.max(axis=-1, keepdims=True)
    e = np.exp(shifted, dtype=np.float32)
    return e / e.sum(axis=-1, keepdims=True, dtype=np.float32)


def reference_fp32(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """FP32 grouped QK, stable softmax, PV (reference.py:47-60). -> [B,Hq,1,D] f32."""
    batch, query_heads, kv_heads, group, _, dim = validate_shapes(q, k, v)
    grouped_q = as_f32(q).reshape(batch, kv_heads, group, dim)
    logits = np.matmul(grouped_q, as_f32(k).transpose(0, 1, 3, 2))
    logits *= np.float32(1.0 / math.sqrt(dim))
    probabilities = _softmax_lastdim(logits)
    output = np.matmul(probabilities, as_f32(v))
    return output.reshape(batch, query_heads, 1, dim).astype(np.float32, copy=False)


def reference(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """reference.py:63-66: FP32 result rounded to BF16 (uint16 bits)."""
    return f32_to_bf16_bits(reference_fp32(q, k, v))


def reference_varlen_fp32(q: np.ndarray, k: np.ndarray, v: np.ndarray, seqlens) -> np.ndarray:
    """Sequence b attends to its first seqlens[b] tokens (clamped to [0, S]).

    Each sequence is exactly reference_fp32 on the sliced cache; an empty
    sequence gives zeros (a matmul over an empty token axis)."""
    batch, query_heads, _, _, length, dim = validate_shapes(q, k, v)
    out = np.zeros((batch, query_heads, 1, dim), dtype=np.float32)
    for b in range(batch):
        n = int(min(max(int(seqlens[b]), 0), length))
        if n == 0:
            continue
        out[b : b + 1] = reference_fp32(q[b : b + 1], k[b : b + 1, :, :n], v[b : b + 1, :, :n])
    return out


# ---------------------------------------------------------------- states
def partial_state(q: np.ndarray, k: np.ndarray, v: np.ndarray, lo: int, hi: int):
    """Unnormalised state over tokens [lo, hi): acc [B,Hq,D], m [B,Hq], l [B,Hq].

    m is the max logit (natural units), l = sum exp(s - m), acc = sum exp(s - m) v.
    An empty range gives acc = 0, m = -inf, l = 0 (csrc/decode.cu:113-131)."""
    batch, query_heads, kv_heads, group, _, dim = validate_shapes(q, k, v)
    if hi <= lo:
        return (
            np.zeros((batch, query_heads, dim), np.float32),
            np.full((batch, query_heads), -np.inf, np.float32),
            np.zeros((batch, query_heads), np.float32),
        )
    grouped_q = as_f32(q).reshape(batch, kv_heads, group, dim)
    kk = as_f32(k)[:, :, lo:hi]
    vv = as_f32(v)[:, :, lo:hi]
    logits = np.matmul(grouped_q, kk.transpose(0, 1, 3, 2)) * np.float32(1.0 / math.sqrt(dim))
    m = logits.max(axis=-1)
    e = np.exp(logits - m[..., None], dtype=np.float32)
    l = e.sum(axis=-1, dtype=np.float32)
    acc = np.matmul(e, vv)
    return (
        acc.reshape(batch, query_heads, dim).astype(np.float32),
        m.reshape(batch, query_heads).astype(np.float32),
        l.reshape(batch, query_heads).astype(np.float32),
    )


def merge_states(accs, ms, ls) -> np.ndarray:
    """merge_splits (csrc/decode.cu:169-184): O = sum e^(m_r-M) acc_r / sum e^(m_r-M) l_r.

    Inputs are stacked over parts on axis 0; rows whose parts are all empty
    give zeros.  Returns float32 with the acc shape minus the part axis."""
    accs = np.asarray(accs, np.float32)
    ms = np.asarray(ms, np.float32)
    ls = np.asarray(ls, np.float32)
    big_m = ms.max(axis=0)
    safe_m = np.where(np.isfinite(big_m), big_m, np.float32(0))
    with np.errstate(invalid="ignore"):
        w = np.where(ls > 0, np.exp(ms - safe_m[None]), np.float32(0)).astype(np.float32)
    num = (w[..., None] * accs).sum(axis=0)
    den = (w * ls).sum(axis=0)
    out = np.zeros_like(num)
    nz = den > 0
    out[nz] = num[nz] / den[nz][..., None]
    return out


def error_metrics(output_bits: np.ndarray, expected_bits: np.ndarray) -> dict:
    """Peak errors in the manner of reference.py:101-121 (1e-6 denominator floor)."""
    out = bf16_bits_to_f32(output_bits)
    exp = bf16_bits_to_f32(expected_bits)
    finite = bool(np.isfinite(out).all())
    diff = np.abs(out - exp)
    return {
        "finite": finite,
        "max_abs_error": float(diff.max()) if diff.size else 0.0,
        "max_rel_error": float((diff / np.maximum(np.abs(exp), 1e-6)).max()) if diff.size else 0.0,
        "allclose": finite and bool(np.all(diff <= ATOL + RTOL * np.abs(exp))),
    }
