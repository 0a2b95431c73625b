"""Per-CTA timeline of back-to-back decode steps (diagnostic build).

    python hpc-ops-sm120_b200/build_lib.py --trace
    python hpc-ops-sm120_b200/trace_decode.py [--config cfg2] [--steps 30] [--fp8]

Loads the diagnostic library (built with -DADB_TRACE into _build/trace/;
the product library is never replaced), runs `--steps` back-to-back decode
steps of a benchmark configuration and prints, for the last launch, where a
step's time goes (globaltimer stamps, microseconds from the moment the
previous grid released this one):

  * producer: first TMA load issued, time spent waiting for free ring stages;
  * consumers (warp 0): first tile arrived, time waiting for full stages,
    time from a full stage to its release (per tile);
  * each CTA's own range done and exit (min / median / max over CTAs), its
    streaming rate (tiles per us) and the time spent merging segments;
  * the gap between the previous grid's last CTA and this grid's release.

The kernels run exactly as in the product build except for the stamps (a few
globaltimer reads per tile), which make steps ~1-3 % slower.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

TRACE_LIB = HERE / "_build" / "trace" / "libattention_decode_b200.so"
TRACE_CTAS = 1024  # adb::kTraceCtas


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--config", default="cfg2")
    parser.add_argument("--steps", type=int, default=30)
    parser.add_argument("--fp8", action="store_true", help="e4m3 K/V cache (per-tensor scales)")
    parser.add_argument("--json", help="also write the raw per-CTA records here")
    args = parser.parse_args()
    if not TRACE_LIB.is_file():
        print(f"{TRACE_LIB} is missing: run `python {HERE / 'build_lib.py'} --trace` first", file=sys.stderr)
        return 2

    import numpy as np
    import torch

    from attention_decode import _lib

    # every ctypes entry point and (by soname) the C++ extension then use the
    # diagnostic library
    _lib.LIB_PATH = TRACE_LIB
    lib = _lib.load_library()
    lib.adb_trace_read.restype = ctypes.c_int
    lib.adb_trace_read.argtypes = [ctypes.c_void_p, ctypes.c_int]
    import attention_decode as ad
    from attention_decode.workloads import BASELINE_CONFIGS

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = BASELINE_CONFIGS[args.config]
    q, k, v, lens = cfg.make_inputs(device, seed=2026)
    if args.fp8:
        ks, vs = float(k.float().abs().max()) / 448.0, float(v.float().abs().max()) / 448.0
        k, v = (k.float() / ks).to(torch.float8_e4m3fn), (v.float() / vs).to(torch.float8_e4m3fn)
        torch.cuda.empty_cache()

        def step():
            return ad.attention_decode_fp8(q, k, v, lens, k_scale=ks, v_scale=vs)
    else:
        def step():
            return ad.attention_decode(q, k, v, lens)

    for _ in range(args.steps):
        step()
    torch.cuda.synchronize(device)
    rec = {}
    for name in ("last", "prev"):
        buf = np.zeros((TRACE_CTAS, 16), dtype=np.uint64)
        nxt = lib.adb_trace_read(buf.ctypes.data, 0)
        lib.adb_trace_read(buf.ctypes.data, (1 - nxt) if name == "last" else nxt)
        rec[name] = buf[: int((buf[:, 1] > 0).sum())].astype(np.int64)
    a, b = rec["last"], rec["prev"]
    t0 = a[:, 2].min()  # release of the grid dependency wait

    def us(x):
        return (x - t0) / 1e3

    tiles = (a[:, 6] & 0xFFFFFFFF) + (a[:, 6] >> 32)
    rate = (a[:, 6] & 0xFFFFFFFF) / np.maximum((a[:, 4] - a[:, 3]) / 1e3, 1e-3)

    def q3(x):
        return [round(float(np.min(x)), 2), round(float(np.median(x)), 2), round(float(np.max(x)), 2)]

    summary = {
        "config": args.config + (" fp8" if args.fp8 else ""),
        "ctas": int(len(a)),
        "producer_first_load_us": q3(us(a[:, 8])),
        "producer_wait_for_free_us": q3(a[:, 10] / 1e3),
        "consumer_first_tile_us": q3(us(a[:, 3])),
        "consumer_wait_full_us": q3(a[:, 11] / 1e3),
        "consumer_busy_ns_per_tile": q3(a[:, 12] / np.maximum(tiles, 1)),
        "own_range_done_us": q3(us(a[:, 4])),
        "cta_exit_us": q3(us(a[:, 5])),
        "tiles_per_us_per_cta": q3(rate),
        "merges": int((a[:, 7] & 0xFFFF).sum()),
        "merge_us_per_cta_max": round(float((a[:, 7] >> 16).max()) / 1e3, 2),
        "previous_grid_last_exit_to_release_us": round(float(t0 - b[:, 5].max()) / 1e3, 2) if len(b) else None,
    }
    print(json.dumps(summary, indent=1))
    if args.json:
        with open(args.json, "w") as fh:
            json.dump({k2: v2.tolist() for k2, v2 in rec.items()}, fh)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
