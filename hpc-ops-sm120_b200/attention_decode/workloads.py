"""Workload contract and reproducible inputs.

``LENGTHS``, ``Workload``, ``all_workloads`` and ``make_inputs`` keep the
reference's first-version contract (attention_decode/workloads.py:9-60): the
56 shapes B in {1,4} x (Hq,Hkv) in {(32,8),(32,32)} x D in {64,128} x T in
LENGTHS.  ``BASELINE_CONFIGS`` adds the five benchmark workloads this build
is measured on (synthetic, seeded; no public dataset is involved):

  cfg1  MHA, CPU-runnable:       B=1   Hq=8  Hkv=8 D=128 S=1024
  cfg2  Llama-3-8B GQA:          B=32  Hq=32 Hkv=8 D=128 S=4096
  cfg3  variable length:         B=64  Hq=32 Hkv=8 D=128 S_b ~ U[1,8192] (1, 7, 8192 forced)
  cfg4  long context, group 8:   B=1   Hq=64 Hkv=8 D=128 S=131072
  cfg5  extreme values, group 8: B=128 Hq=64 Hkv=8 D=128 S=16384, K ~ N(0,8^2)
                                 with one key per (b, kv_head) scaled x50

Algorithmic bytes of one decode step count each valid K and V element once
plus the Q read and the O write: 2*2*D*Hkv*sum_b(S_b) + 2*2*B*Hq*D.
"""

from __future__ import annotations

from dataclasses import dataclass
from itertools import product

import torch

LENGTHS = (1, 127, 128, 129, 512, 2048, 8192)


@dataclass(frozen=True)
class Workload:
    batch: int
    query_heads: int
    kv_heads: int
    head_dim: int
    sequence_length: int

    @property
    def key(self) -> str:
        return (
            f"b{self.batch}_hq{self.query_heads}_hkv{self.kv_heads}"
            f"_d{self.head_dim}_t{self.sequence_length}"
        )

    @property
    def q_shape(self) -> tuple[int, ...]:
        return (self.batch, self.query_heads, 1, self.head_dim)

    @property
    def kv_shape(self) -> tuple[int, ...]:
        return (self.batch, self.kv_heads, self.sequence_length, self.head_dim)

    @property
    def kv_bytes(self) -> int:
        return 2 * 2 * self.batch * self.kv_heads * self.sequence_length * self.head_dim


def all_workloads() -> tuple[Workload, ...]:
    """All 56 contract shapes in a stable order (reference workloads.py:40-47)."""
    return tuple(
        Workload(batch, query_heads, kv_heads, head_dim, length)
        for batch, (query_heads, kv_heads), head_dim, length in product(
            (1, 4), ((32, 8), (32, 32)), (64, 128), LENGTHS
        )
    )


def make_inputs(workload: Workload, *, device="cuda", seed: int = 2026):
    """Contiguous BF16 tensors from a private generator (reference workloads.py:50-60)."""
    generator = torch.Generator(device=device).manual_seed(seed)
    kwargs = {"device": device, "dtype": torch.bfloat16, "generator": generator}
    return (
        torch.randn(workload.q_shape, **kwargs),
        torch.randn(workload.kv_shape, **kwargs),
        torch.randn(workload.kv_shape, **kwargs),
    )


@dataclass(frozen=True)
class BaselineConfig:
    name: str
    batch: int
    query_heads: int
    kv_heads: int
    head_dim: int
    kv_len: int
    varlen: bool = False
    extreme: bool = False
    description: str = ""

    @property
    def group(self) -> int:
        return self.query_heads // self.kv_heads

    def algorithmic_bytes(self, seqlens=None) -> int:
        """K+V bytes of valid tokens + Q read + O write (bf16)."""
        if seqlens is None:
            tokens = self.batch * self.kv_len
        else:
            tokens = int(torch.as_tensor(seqlens).clamp(0, self.kv_len).sum().item())
        return 2 * 2 * self.head_dim * self.kv_heads * tokens + 2 * 2 * self.batch * self.query_heads * self.head_dim

    def as_dict(self) -> dict:
        return {
            "workload": self.name,
            "batch": self.batch,
            "q_heads": self.query_heads,
            "kv_heads": self.kv_heads,
            "head_dim": self.head_dim,
            "kv_len": self.kv_len,
            "varlen": self.varlen,
            "extreme_values": self.extreme,
        }

    def make_seqlens(self, seed: int) -> torch.Tensor | None:
        """Seeded lengths ~ U[1, S] with 1, 7 and S forced in at seeded positions."""
        if not self.varlen:
            return None
        generator = torch.Generator(device="cpu").manual_seed(seed + 7919)
        lens = torch.randint(1, self.kv_len + 1, (self.batch,), generator=generator, dtype=torch.int64)
        positions = torch.randperm(self.batch, generator=generator)[:3]
        lens[positions] = torch.tensor([1, 7, self.kv_len])
        return lens.to(torch.int32)

    def make_inputs(self, device, seed: int = 2026, batch_slice=None):
        """(q, k, v, seqlens) on `device`.  K/V are generated directly on the
        device (seeded); ``batch_slice`` (a slice or a list of sequence
        indices) selects a subset of the sequences (batch sharding) with
        identical values to the full batch."""
        device = torch.device(device)
        seqlens = self.make_seqlens(seed)
        if batch_slice is None:
            rows = list(range(self.batch))
        elif isinstance(batch_slice, slice):
            rows = list(range(self.batch)[batch_slice])
        else:
            rows = [int(b) for b in batch_slice]
        q_full = torch.randn(
            (self.batch, self.query_heads, 1, self.head_dim),
            generator=torch.Generator(device="cpu").manual_seed(seed),
            dtype=torch.float32,
        ).to(torch.bfloat16)
        q = q_full[rows].contiguous().to(device)
        kv_shape = (len(rows), self.kv_heads, self.kv_len, self.head_dim)
        k = torch.empty(kv_shape, dtype=torch.bfloat16, device=device)
        v = torch.empty(kv_shape, dtype=torch.bfloat16, device=device)
        std = 8.0 if self.extreme else 1.0
        for i, b in enumerate(rows):
            # one generator per sequence: a shard reproduces the full batch's values
            gen = torch.Generator(device=device).manual_seed(seed * 1_000_003 + b)
            k[i].normal_(0.0, std, generator=gen)
            v[i].normal_(0.0, 1.0, generator=gen)
            if self.extreme:
                spike = torch.randint(0, self.kv_len, (self.kv_heads,), generator=gen, device=device)
                heads = torch.arange(self.kv_heads, device=device)
                k[i, heads, spike] *= 50
        if seqlens is not None:
            seqlens = seqlens[rows].contiguous().to(device)
        return q, k, v, seqlens


BASELINE_CONFIGS = {
    "cfg1": BaselineConfig("cfg1", 1, 8, 8, 128, 1024, description="MHA, CPU-runnable FP32 reference decode"),
    "cfg2": BaselineConfig("cfg2", 32, 32, 8, 128, 4096, description="Llama-3-8B-shaped GQA decode"),
    "cfg3": BaselineConfig("cfg3", 64, 32, 8, 128, 8192, varlen=True, description="variable-length batch decode"),
    "cfg4": BaselineConfig("cfg4", 1, 64, 8, 128, 131072, description="long-context split-K decode, group 8"),
    "cfg5": BaselineConfig(
        "cfg5", 128, 64, 8, 128, 16384, extreme=True, description="numerically extreme large-batch decode"
    ),
}
