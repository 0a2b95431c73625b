"""Generate tests/golden/golden_vectors.npz by running the REFERENCE's own FP32
oracle (attention_decode/reference.py: reference_fp32 / reference) on the
inputs of tests/golden/cases.py.

Usage (needs a checkout of the reference repository and torch on CPU):

    python tests/golden/make_golden.py --reference-root <path to reference checkout>

For each case the file stores the SHA-256 of the generated inputs and the
reference's FP32 output and BF16-rounded output (as uint16 bits).  Variable
length cases run the reference per sequence on the sliced cache (the
reference has no seqlens argument).  Only this script imports the reference;
the tests read the .npz.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference-root", required=True, help="checkout of the reference repository")
    parser.add_argument("--output", default=None)
    args = parser.parse_args()

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.abspath(args.reference_root))
    import torch
    from attention_decode.reference import reference, reference_fp32  # the reference's oracle

    from cases import CASES, GOLDEN_PATH

    def to_torch(bits):
        return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)

    payload = {}
    for case in CASES:
        q, k, v, lens = case.inputs()
        tq, tk, tv = to_torch(q), to_torch(k), to_torch(v)
        if lens is None:
            out32 = reference_fp32(tq, tk, tv)
            out16 = reference(tq, tk, tv)
        else:
            out32 = torch.zeros(q.shape, dtype=torch.float32)
            for b, n in enumerate(lens.tolist()):
                n = min(max(n, 0), case.length)
                if n:
                    out32[b : b + 1] = reference_fp32(
                        tq[b : b + 1], tk[b : b + 1, :, :n].contiguous(), tv[b : b + 1, :, :n].contiguous()
                    )
            out16 = out32.to(torch.bfloat16)
        payload[f"{case.name}/checksum"] = np.frombuffer(bytes.fromhex(case.checksum()), dtype=np.uint8)
        payload[f"{case.name}/out_fp32"] = out32.numpy().astype(np.float32)
        payload[f"{case.name}/out_bf16"] = out16.view(torch.int16).numpy().view(np.uint16)
        print(f"{case.name:24s} out {tuple(out32.shape)} finite={bool(torch.isfinite(out32).all())}")
    target = args.output or GOLDEN_PATH
    np.savez_compressed(target, **payload)
    print(f"wrote {target} ({os.path.getsize(target)} bytes)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
