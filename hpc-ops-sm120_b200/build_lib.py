"""Build libattention_decode_b200.so in-tree with nvcc for sm_100a.

    python hpc-ops-sm120_b200/build_lib.py [--force] [--verbose]

The library is one translation unit (csrc/decode_capi.cu) with the CUDA
runtime linked statically and the driver's tensor-map encoder fetched at run
time, so it depends on nothing but libc/libstdc++ and loads on machines
without a GPU.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
ROOT = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = ROOT / "include"
OUTPUT = PACKAGE_DIR / "attention_decode" / "libattention_decode_b200.so"
SOURCES = [CSRC / "decode_capi.cu"]
DEPENDENCIES = SOURCES + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-shared",
    "-cudart", "static",
]


def nvcc_path() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.is_file():
        return str(candidate)
    raise RuntimeError("nvcc not found (set CUDA_HOME or put nvcc on PATH)")


def up_to_date() -> bool:
    if not OUTPUT.is_file():
        return False
    built = OUTPUT.stat().st_mtime
    return all(dep.stat().st_mtime <= built for dep in DEPENDENCIES)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUTPUT
    cmd = [nvcc_path(), *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", *map(str, SOURCES), "-o", str(OUTPUT) + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=not verbose, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    os.replace(str(OUTPUT) + ".tmp", OUTPUT)
    return OUTPUT


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
