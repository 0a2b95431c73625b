"""Build the reference's own CUDA kernel for B200, as a comparison baseline.

    python baseline/build_ref_kernel.py --reference-root <reference checkout>

The reference builds its extension for sm_120 only (attention_decode/__init__.py:21)
and refuses any other compute capability at run time (csrc/decode.cu:244).  To
time it on B200 this script copies its two sources (csrc/binding.cpp,
csrc/decode.cu) into baseline/_ref/src (git-ignored, never committed), changes
exactly two things -- the capability gate now accepts 10.x, and the code is
generated for sm_100a -- and builds them with torch.utils.cpp_extension into
baseline/_ref/build/attention_decode_ref_sm100.so.  Nothing else of the kernel
changes, so its limits stay: GQA groups 1 and 4, no sequence lengths, at most
INT_MAX elements per tensor (of the BASELINE configs only cfg1 and cfg2 run).

bench.py --impl ref-kernel loads the built module directly (no rebuild on the
GPU machine).
"""

from __future__ import annotations

import argparse
import os
import re
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
MODULE = "attention_decode_ref_sm100"
GATE = re.compile(r"properties->major == 12 && properties->minor == 0")


def module_path() -> Path:
    return OUT / "build" / f"{MODULE}.so"


def build(reference_root: str, verbose: bool = False) -> Path:
    src_dir = Path(reference_root) / "csrc"
    dst = OUT / "src"
    dst.mkdir(parents=True, exist_ok=True)
    shutil.copyfile(src_dir / "binding.cpp", dst / "binding.cpp")
    text = (src_dir / "decode.cu").read_text()
    patched, n = GATE.subn("properties->major == 10", text)
    if n != 1:
        raise RuntimeError("capability gate not found in csrc/decode.cu; the reference changed")
    (dst / "decode.cu").write_text(patched)
    build_dir = OUT / "build"
    build_dir.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils.cpp_extension import load

    load(
        name=MODULE,
        sources=[str(dst / "binding.cpp"), str(dst / "decode.cu")],
        build_directory=str(build_dir),
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", "-lineinfo", "-gencode=arch=compute_100a,code=sm_100a"],
        verbose=verbose,
    )
    return module_path()


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference-root", required=True)
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(args.reference_root, args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
