"""Decode over a paged KV cache (block table), both page layouts, against the
CPU oracle on the same tokens gathered into a contiguous cache, and against
the contiguous entry point.  Pages are scattered at random block ids, the
unused slots of each sequence's last page and every unused block hold NaN,
and block-table entries past a sequence's last page are out of range: none of
them may reach the output."""

from __future__ import annotations

import math

import pytest
import torch

import attention_decode as ad
from helpers import check, oracle_reference

pytestmark = pytest.mark.gpu


def make_paged(device, lengths, hq, hkv, dim, page, layout, seed, spare_blocks=3):
    gen = torch.Generator(device="cpu").manual_seed(seed)
    batch = len(lengths)
    pages = [max(1, math.ceil(n / page)) for n in lengths]
    max_blocks = max(pages) + 1
    cap = max_blocks * page
    q = torch.randn((batch, hq, 1, dim), generator=gen).to(torch.bfloat16)
    k = torch.randn((batch, hkv, cap, dim), generator=gen).to(torch.bfloat16)
    v = torch.randn((batch, hkv, cap, dim), generator=gen).to(torch.bfloat16)
    for b, n in enumerate(lengths):
        k[b, :, n:] = float("nan")
        v[b, :, n:] = float("nan")
    total = sum(pages) + spare_blocks
    perm = torch.randperm(total, generator=gen).tolist()
    shape = (total, hkv, page, dim) if layout == "HND" else (total, page, hkv, dim)
    k_cache = torch.full(shape, float("nan"), dtype=torch.bfloat16)
    v_cache = torch.full(shape, float("nan"), dtype=torch.bfloat16)
    table = torch.full((batch, max_blocks), 10**6, dtype=torch.int32)  # out of range past the end
    b_idx = torch.tensor([b for b in range(batch) for _ in range(pages[b])])
    j_idx = torch.tensor([j for b in range(batch) for j in range(pages[b])])
    blk = torch.tensor(perm[: len(b_idx)])
    table[b_idx, j_idx] = blk.to(torch.int32)
    for src, dst in ((k, k_cache), (v, v_cache)):
        by_page = src.view(batch, hkv, max_blocks, page, dim).permute(0, 2, 1, 3, 4)  # [B, blocks, hkv, page, dim]
        chosen = by_page[b_idx, j_idx]  # [n, hkv, page, dim]
        dst[blk] = chosen if layout == "HND" else chosen.transpose(1, 2)
    lens = torch.tensor(lengths, dtype=torch.int32)
    to = lambda t: t.to(device)  # noqa: E731
    return to(q), to(k), to(v), to(k_cache), to(v_cache), to(table), to(lens)


@pytest.mark.parametrize("layout", ("HND", "NHD"))
@pytest.mark.parametrize("page", (8, 16, 64, 128, 256))
@pytest.mark.parametrize("dim,hq,hkv", ((128, 32, 8), (64, 32, 32), (128, 64, 8)))
def test_paged_matches_oracle(layout, page, dim, hq, hkv, device, record_property):
    lengths = [1, page - 1, page, page + 1, 3 * page + 5, 0, 1000, 2 * page]
    q, k, v, kc, vc, table, lens = make_paged(device, lengths, hq, hkv, dim, page, layout, seed=page + dim)
    out = ad.attention_decode_paged(q, kc, vc, table, lens, layout=layout)
    check(out, oracle_reference(q, k, v, lens), q, record_property)
    contiguous = ad.attention_decode(q, k, v, lens)
    check(out, contiguous, q, None, atol=1e-2, rtol=2.0**-7)


@pytest.mark.parametrize("layout", ("HND", "NHD"))
def test_paged_long_sequences_split_across_ctas(layout, device, record_property):
    lengths = [20000, 7, 16384, 9000]
    q, k, v, kc, vc, table, lens = make_paged(device, lengths, 64, 8, 128, 16, layout, seed=77)
    out = ad.attention_decode_paged(q, kc, vc, table, lens, layout=layout)
    check(out, oracle_reference(q, k, v, lens), q, record_property)
    again = ad.attention_decode_paged(q, kc, vc, table, lens, layout=layout)
    check(again, out, q, None, atol=1e-3, rtol=2.0**-7)


def test_paged_rejects_bad_arguments(device):
    q, k, v, kc, vc, table, lens = make_paged(device, [5, 9], 32, 8, 128, 16, "HND", seed=3)
    with pytest.raises(ValueError):
        ad.attention_decode_paged(q, kc, vc, table, lens, layout="BHSD")
    with pytest.raises(RuntimeError, match="int32"):
        ad.attention_decode_paged(q, kc, vc, table.long(), lens)
    with pytest.raises(RuntimeError, match="power of two"):
        odd = torch.zeros((4, 8, 12, 128), dtype=torch.bfloat16, device=device)
        ad.attention_decode_paged(q, odd, odd, table, lens)
