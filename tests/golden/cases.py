"""Golden-vector cases: deterministic inputs for pinning the CPU oracle and
the CUDA kernels against the reference's own FP32 oracle.

Inputs are generated here with numpy's PCG64 stream and rounded to BF16 bit
patterns (uint16), so the same arrays can be rebuilt on any machine from the
seed alone; ``golden_vectors.npz`` stores only a checksum of each case's
inputs and the reference's outputs.  The shapes and special constructions
follow the reference's own tests:

  gqa_formula        tests/test_attention_decode.py:228-239
  single_token_*     tests/test_attention_decode.py:156-165 (T=1 returns V)
  mma_pad_*          tests/test_attention_decode.py:105-110
  split_*            tests/test_attention_decode.py:96-102
  separated_maxima   tests/test_attention_decode.py:113-132
  common_offset      tests/test_attention_decode.py:195-204
  large_logits_*     tests/test_attention_decode.py:184-192
  gqa_grouping       tests/test_attention_decode.py:168-181
  odd_heads_*        tests/test_extreme_decode.py:196-207
plus the BASELINE workload shapes at small size (MHA cfg1 exactly, group-8,
the extreme-value K distribution with a x50 spike, and variable lengths).
"""

from __future__ import annotations

import hashlib
import os
import sys
from dataclasses import dataclass, field

import numpy as np

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from oracle.attention_decode_oracle import bf16_bits_to_f32, f32_to_bf16_bits  # noqa: E402


def randn_bf16(rng: np.random.Generator, shape, scale: float = 1.0) -> np.ndarray:
    """N(0, scale^2) samples rounded to BF16 bits."""
    return f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale))


def const_bf16(shape, value: float) -> np.ndarray:
    return np.full(shape, f32_to_bf16_bits(np.array([value], np.float32))[0], dtype=np.uint16)


@dataclass
class Case:
    name: str
    batch: int
    q_heads: int
    kv_heads: int
    length: int
    dim: int
    seed: int
    kind: str = "random"
    seqlens: tuple = field(default=())

    def inputs(self):
        """(q, k, v) as uint16 BF16 bits, plus seqlens (or None)."""
        rng = np.random.default_rng(self.seed)
        q_shape = (self.batch, self.q_heads, 1, self.dim)
        kv_shape = (self.batch, self.kv_heads, self.length, self.dim)
        q = randn_bf16(rng, q_shape)
        k = randn_bf16(rng, kv_shape)
        v = randn_bf16(rng, kv_shape)
        group = self.q_heads // self.kv_heads
        if self.kind == "scaled32":
            q = f32_to_bf16_bits(bf16_bits_to_f32(q) * 32)
            k = f32_to_bf16_bits(bf16_bits_to_f32(k) * 32)
        elif self.kind == "separated_maxima":
            q = const_bf16(q_shape, 1.0)
            q[:, 1::2] = const_bf16((1,), -1.0)[0]
            k[:, :, :256] = const_bf16((1,), -32.0)[0]
            k[:, :, 256:512] = const_bf16((1,), 0.0)[0]
            k[:, :, 512:] = const_bf16((1,), 32.0)[0]
            values = np.arange(self.kv_heads, dtype=np.float32) / 8 + 0.125
            v = np.broadcast_to(
                f32_to_bf16_bits(values).reshape(1, self.kv_heads, 1, 1), kv_shape
            ).copy()
        elif self.kind == "common_offset":
            q = const_bf16(q_shape, 32.0)
            k = const_bf16(kv_shape, 32.0)
        elif self.kind == "gqa_grouping":
            q = const_bf16(q_shape, 0.0)
            k = const_bf16(kv_shape, 0.0)
            values = (
                np.arange(self.batch, dtype=np.float32).reshape(-1, 1) * 8
                + np.arange(self.kv_heads, dtype=np.float32).reshape(1, -1)
            )
            v = np.broadcast_to(
                f32_to_bf16_bits(values).reshape(self.batch, self.kv_heads, 1, 1), kv_shape
            ).copy()
        elif self.kind == "extreme":
            # K ~ N(0, 8^2) and one key per (b, kv_head) scaled x50 (BASELINE cfg5 law).
            k = randn_bf16(rng, kv_shape, 8.0)
            spike = rng.integers(0, self.length, size=(self.batch, self.kv_heads))
            kf = bf16_bits_to_f32(k)
            for b in range(self.batch):
                for h in range(self.kv_heads):
                    kf[b, h, spike[b, h]] *= 50
            k = f32_to_bf16_bits(kf)
        del group
        lens = np.array(self.seqlens, dtype=np.int32) if self.seqlens else None
        return q, k, v, lens

    def checksum(self) -> str:
        q, k, v, lens = self.inputs()
        h = hashlib.sha256()
        for a in (q, k, v) + ((lens,) if lens is not None else ()):
            h.update(np.ascontiguousarray(a).tobytes())
        return h.hexdigest()


CASES = [
    Case("gqa_formula", 1, 32, 8, 127, 64, 101),
    Case("single_token_d64", 4, 32, 8, 1, 64, 102, "scaled32"),
    Case("single_token_d128_mha", 4, 32, 32, 1, 128, 103, "scaled32"),
    Case("mma_pad_t2", 1, 32, 8, 2, 64, 104),
    Case("mma_pad_t15", 1, 32, 8, 15, 64, 105),
    Case("mma_pad_t16_mha", 1, 32, 32, 16, 128, 106),
    Case("mma_pad_t17_mha", 1, 32, 32, 17, 128, 107),
    Case("split_255", 1, 32, 8, 255, 128, 108),
    Case("split_256", 1, 32, 8, 256, 128, 109),
    Case("split_257_mha", 1, 32, 32, 257, 64, 110),
    Case("separated_maxima", 1, 32, 8, 513, 64, 111, "separated_maxima"),
    Case("common_offset", 1, 32, 8, 129, 64, 112, "common_offset"),
    Case("large_logits_x32", 1, 32, 8, 129, 128, 113, "scaled32"),
    Case("gqa_grouping", 4, 32, 8, 127, 64, 114, "gqa_grouping"),
    Case("odd_heads_h12", 1, 12, 3, 129, 128, 115),
    Case("odd_heads_h7", 4, 7, 7, 129, 64, 116),
    Case("mha_cfg1", 1, 8, 8, 1024, 128, 117),
    Case("group8", 1, 64, 8, 300, 128, 118),
    Case("group8_d64", 2, 64, 8, 77, 64, 119),
    Case("extreme_spike", 2, 64, 8, 512, 128, 120, "extreme"),
    Case("varlen", 4, 32, 8, 300, 128, 121, "random", (1, 7, 300, 150)),
    Case("varlen_group8", 3, 64, 8, 200, 64, 122, "random", (200, 1, 65)),
]

CASES_BY_NAME = {c.name: c for c in CASES}
GOLDEN_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_vectors.npz")
