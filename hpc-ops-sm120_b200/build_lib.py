"""Build libattention_decode_b200.so in-tree with nvcc for sm_100a, and the
PyTorch C++ extension adb_torch_ext.so over it.

    python hpc-ops-sm120_b200/build_lib.py [--force] [--verbose]

The library is one translation unit (csrc/decode_capi.cu) with the CUDA
runtime linked statically and the driver's tensor-map encoder fetched at run
time, so it depends on nothing but libc/libstdc++ and loads on machines
without a GPU.  The extension (csrc/torch_binding.cpp) holds no kernels: it
is the reference's pybind `forward` (csrc/binding.cpp:3-8) over the C ABI,
compiled with g++ against torch's headers and linked to the library, which it
finds next to itself (rpath $ORIGIN).
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
    "-Xlinker", "-soname=libattention_decode_b200.so",
]

TORCH_EXT_NAME = "adb_torch_ext"
TORCH_EXT_SOURCE = CSRC / "torch_binding.cpp"
TORCH_EXT_OUTPUT = PACKAGE_DIR / "attention_decode" / f"{TORCH_EXT_NAME}.so"


def nvcc_path() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.is_file():
        return str(candidate)
    raise RuntimeError("nvcc not found (set CUDA_HOME or put nvcc on PATH)")


def up_to_date(output: Path = OUTPUT, dependencies=None) -> bool:
    if not output.is_file():
        return False
    built = output.stat().st_mtime
    return all(dep.stat().st_mtime <= built for dep in (dependencies or DEPENDENCIES))


# Diagnostic build: the same library with the per-CTA timeline compiled in
# (-DADB_TRACE), written outside the package (git-ignored _build/); used by
# trace_decode.py.  The product never loads it.
TRACE_OUTPUT = PACKAGE_DIR / "_build" / "trace" / "libattention_decode_b200.so"


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> Path:
    output = TRACE_OUTPUT if trace else OUTPUT
    if not force and up_to_date(output):
        return output
    output.parent.mkdir(parents=True, exist_ok=True)
    extra = ["-DADB_TRACE"] if trace else []
    cmd = [nvcc_path(), *NVCC_FLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", *map(str, SOURCES), "-o", str(output) + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=not verbose, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    os.replace(str(output) + ".tmp", output)
    return output


def build_torch_extension(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/torch_binding.cpp into attention_decode/adb_torch_ext.so
    (needs the library built first)."""
    deps = [TORCH_EXT_SOURCE, INCLUDE / "attention_decode_b200.h", OUTPUT]
    if not force and up_to_date(TORCH_EXT_OUTPUT, deps):
        return TORCH_EXT_OUTPUT
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    includes = cpp_extension.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], str(INCLUDE)]
    libdirs = cpp_extension.library_paths(device_type="cuda")
    cxx = os.environ.get("CXX", "g++")
    cmd = [
        cxx, "-shared", "-fPIC", "-O3", "-std=c++17", "-fvisibility=hidden",
        f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
        "-DTORCH_API_INCLUDE_EXTENSION_H", f"-DTORCH_EXTENSION_NAME={TORCH_EXT_NAME}",
        *[f"-I{p}" for p in includes],
        str(TORCH_EXT_SOURCE),
        f"-L{OUTPUT.parent}", "-l:libattention_decode_b200.so", "-Wl,-rpath,$ORIGIN",
        *[f"-L{p}" for p in libdirs],
        "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart",
        "-o", str(TORCH_EXT_OUTPUT) + ".tmp",
    ]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=not verbose, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"{cxx} failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    os.replace(str(TORCH_EXT_OUTPUT) + ".tmp", TORCH_EXT_OUTPUT)
    return TORCH_EXT_OUTPUT


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--trace", action="store_true", help="build only the diagnostic (per-CTA timeline) library")
    args = parser.parse_args()
    if args.trace:
        print(build(force=args.force, verbose=args.verbose, trace=True))
        return 0
    print(build(force=args.force, verbose=args.verbose))
    print(build_torch_extension(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
