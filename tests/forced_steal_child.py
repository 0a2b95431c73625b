"""Child process of tests/test_load_balancing.py.

The library reads its load-balancing knobs (ADB_MAX_STEALS, ADB_CLAIM_DIVISOR)
once per process, so the parent starts this script with them set.  It decodes
a fixed list of seeded cases several times each (the steals, and so the
segment boundaries, differ from call to call), checks every result against the
CPU oracle, and prints one JSON line per case.
"""

from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for path in (ROOT, os.path.join(ROOT, "hpc-ops-sm120_b200"), HERE):
    if path not in sys.path:
        sys.path.insert(0, path)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import attention_decode as ad  # noqa: E402
from helpers import ATOL, RTOL, inputs, oracle_reference  # noqa: E402

# (name, batch, q_heads, kv_heads, kv_len, head_dim, lengths or None)
CASES = [
    ("uniform_d128_g4", 4, 32, 8, 16385, 128, None),
    ("uniform_d64_g1", 2, 32, 32, 8193, 64, None),
    ("uniform_d128_g8_long", 1, 64, 8, 131073, 128, None),
    ("varlen_d128_g8", 12, 64, 8, 24576, 128, (24576, 1, 0, 9000, 24575, 129, 7, 20000, 128, 16384, 3, 24000)),
    ("varlen_d64_g4", 8, 32, 8, 20000, 64, (19999, 20000, 1, 5000, 0, 12345, 256, 17)),
]
REPEATS = 4


def run_case(index, name, batch, hq, hkv, length, dim, lengths, device):
    q, k, v = inputs(device, length, dim, hkv, batch=batch, hq=hq, seed=4100 + index)
    seqlens = None
    if lengths is not None:
        seqlens = torch.tensor(lengths, dtype=torch.int32, device=device)
        for b, n in enumerate(lengths):
            k[b, :, n:] = float("nan")  # padding must never reach the output
            v[b, :, n:] = float("nan")
    expected = oracle_reference(q, k, v, seqlens).float()
    worst_abs, worst_excess, finite = 0.0, -1.0, True
    for _ in range(REPEATS):
        out = ad.attention_decode(q, k, v, seqlens).float()
        finite &= bool(torch.isfinite(out).all().item())
        err = (out - expected).abs()
        worst_abs = max(worst_abs, err.max().item())
        worst_excess = max(worst_excess, (err - (ATOL + RTOL * expected.abs())).max().item())
    acc, ml = ad.attention_decode_partial(q, k, v, seqlens)
    merged = ad.combine_partials(acc.reshape(1, -1, dim), ml.reshape(1, -1, 2)).float().reshape(expected.shape)
    partial_excess = ((merged - expected).abs() - (ATOL + RTOL * expected.abs())).max().item()
    torch.cuda.synchronize(device)
    return {
        "case": name,
        "finite": finite,
        "max_abs": worst_abs,
        "excess": worst_excess,
        "partial_excess": partial_excess,
        "error_flag": ad.read_error_flag(device.index or 0),
    }


def run_paged_case(device):
    """A paged cache (16-token pages at shuffled block ids) with stealing on."""
    from test_paged import make_paged

    lengths = [30000, 5, 24000, 17, 9000, 31000]
    q, k, v, kc, vc, table, lens = make_paged(device, lengths, 64, 8, 128, 16, "NHD", seed=4242)
    expected = oracle_reference(q, k, v, lens).float()
    worst_excess, finite = -1.0, True
    for _ in range(REPEATS):
        out = ad.attention_decode_paged(q, kc, vc, table, lens, layout="NHD").float()
        finite &= bool(torch.isfinite(out).all().item())
        worst_excess = max(worst_excess, ((out - expected).abs() - (ATOL + RTOL * expected.abs())).max().item())
    torch.cuda.synchronize(device)
    return {"case": "paged_nhd_p16", "finite": finite, "max_abs": None, "excess": worst_excess,
            "partial_excess": -1.0, "error_flag": ad.read_error_flag(device.index or 0)}


def run_append_case(device):
    """Decode with an appended token, stealing on: output and cache write."""
    lengths = [20000, 3, 16000, 0, 12000]
    batch, hkv, cap, dim = len(lengths), 8, 20480, 128
    q, k, v = inputs(device, cap, dim, hkv, batch=batch, hq=64, seed=4343)
    k_new = k[:, :, :1].flip(0).contiguous()
    v_new = v[:, :, :1].flip(0).contiguous()
    lens = torch.tensor(lengths, dtype=torch.int32, device=device)
    k2, v2 = k.clone(), v.clone()
    for b, n in enumerate(lengths):
        k2[b, :, n] = k_new[b, :, 0]
        v2[b, :, n] = v_new[b, :, 0]
    expected = oracle_reference(q, k2, v2, lens + 1).float()
    out = ad.attention_decode_append(q, k_new, v_new, k, v, lens).float()
    torch.cuda.synchronize(device)
    excess = ((out - expected).abs() - (ATOL + RTOL * expected.abs())).max().item()
    cache_ok = bool(torch.equal(k, k2) and torch.equal(v, v2))
    return {"case": "append", "finite": bool(torch.isfinite(out).all().item()) and cache_ok, "max_abs": None,
            "excess": excess, "partial_excess": -1.0, "error_flag": ad.read_error_flag(device.index or 0)}


def main() -> int:
    device = torch.device("cuda", 0)
    for index, case in enumerate(CASES):
        print(json.dumps(run_case(index, *case, device=device)), flush=True)
    print(json.dumps(run_paged_case(device)), flush=True)
    print(json.dumps(run_append_case(device)), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
