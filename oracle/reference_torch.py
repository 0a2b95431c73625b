"""Torch-on-CPU restatement of the reference's FP32 decode -- TEST
INFRASTRUCTURE and CPU BASELINE.

Only tests/ and bench.py (its CPU-baseline leg and its ``--impl reference``
arm) use this module: it is the reference's own CPU algorithm timed on the
host cores, never part of the product path.

The reference's CPU path is ``reference_fp32`` (attention_decode/reference.py:47-60),
written in torch.  This module makes the same torch calls in the same order,
so that its speed on a given host is the reference's speed there (the numpy
restatement in attention_decode_oracle.py is the pinned checker but runs
slower than torch's CPU kernels):

    grouped_q = q.float().reshape(B, Hkv, G, D)                 # :55
    logits    = torch.matmul(grouped_q, k.float().transpose(-1, -2))   # :56
    logits.mul_(1 / sqrt(D))                                    # :57
    probs     = torch.softmax(logits, dim=-1, dtype=float32)    # :58
    out       = torch.matmul(probs, v.float())                  # :59
    return out.reshape(B, Hq, 1, D)                             # :60

The reference module itself does not exist on the machine that runs the
benchmark, which is why it is restated here.  Pinning:
tests/test_oracle_golden.py checks this module against the golden outputs the
reference's reference.py produced (tests/golden/golden_vectors.npz).
"""

from __future__ import annotations

import math

import torch


@torch.no_grad()
def reference_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """FP32 grouped QK, stable softmax and PV of BF16 (or FP32) CPU tensors."""
    batch, query_heads, _, dim = q.shape
    kv_heads = k.shape[1]
    group = query_heads // kv_heads
    grouped_q = q.float().reshape(batch, kv_heads, group, dim)
    logits = torch.matmul(grouped_q, k.float().transpose(-1, -2))
    logits.mul_(1.0 / math.sqrt(dim))
    probabilities = torch.softmax(logits, dim=-1, dtype=torch.float32)
    output = torch.matmul(probabilities, v.float())
    return output.reshape(batch, query_heads, 1, dim)


@torch.no_grad()
def reference_varlen_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seqlens) -> torch.Tensor:
    """Sequence b attends to its first seqlens[b] tokens (clamped to [0, S]);
    each sequence is reference_fp32 on the sliced cache, an empty one gives
    zeros.  The reference has no lengths; this is its computation per slice."""
    batch, query_heads, _, dim = q.shape
    length = k.shape[2]
    out = torch.zeros((batch, query_heads, 1, dim), dtype=torch.float32)
    for b in range(batch):
        n = int(min(max(int(seqlens[b]), 0), length))
        if n:
            out[b : b + 1] = reference_fp32(q[b : b + 1], k[b : b + 1, :, :n], v[b : b + 1, :, :n])
    return out
