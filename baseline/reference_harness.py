"""Run the reference's own tests and benchmark, unmodified, against this package.

    python baseline/reference_harness.py prepare --reference-root <checkout>
    python baseline/reference_harness.py tests      [pytest args...]
    python baseline/reference_harness.py benchmark  [bench_attention_decode.py args...]

`prepare` copies, byte for byte, the reference's tests/test_attention_decode.py,
tests/test_extreme_decode.py, benchmarks/bench_attention_decode.py, pytest.ini
and attention_decode/reference.py into baseline/_ref/harness/ (git-ignored,
never committed).  `tests` and `benchmark` then run those files in a
subprocess where ``import attention_decode`` is THIS package
(hpc-ops-sm120_b200/attention_decode, whose ``attention_decode`` is the
extension's ``forward``) and ``attention_decode.reference`` is the
reference's own reference.py (registered by baseline/reference_harness_plugin.py),
so their FP32 oracle, SDPA and FA2 baselines are the reference's code.
``attention_decode.workloads`` is this package's copy of the reference's
workload contract (attention_decode/workloads.py:9-60).

The two documented differences, and nothing else:
  * the capability gate: the reference's fixtures skip unless
    torch.cuda.get_device_capability() == (12, 0) (tests/test_attention_decode.py:36-42,
    tests/test_extreme_decode.py:16-19); for the test run the plugin reports
    (12, 0) on a compute-capability 10.x device;
  * test_rejects_unsupported_gqa_group[4] (a GQA group of 8 must be rejected,
    tests/test_attention_decode.py:320-324) is deselected: this build
    supports group 8 on purpose (the benchmark configurations need it).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
PACKAGE_DIR = ROOT / "hpc-ops-sm120_b200"
HARNESS = HERE / "_ref" / "harness"
FILES = (
    "tests/test_attention_decode.py",
    "tests/test_extreme_decode.py",
    "benchmarks/bench_attention_decode.py",
    "pytest.ini",
    "attention_decode/reference.py",
)
DESELECT = ("tests/test_attention_decode.py::test_rejects_unsupported_gqa_group[4]",)


def prepare(reference_root: str | os.PathLike) -> Path:
    src = Path(reference_root)
    for rel in FILES:
        dst = HARNESS / ("reference.py" if rel.endswith("reference.py") else rel)
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(src / rel, dst)
    return HARNESS


def ready() -> bool:
    return all((HARNESS / ("reference.py" if r.endswith("reference.py") else r)).is_file() for r in FILES)


def _env() -> dict:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(HERE), str(PACKAGE_DIR), env.get("PYTHONPATH", "")]).rstrip(os.pathsep)
    env["ADB_REFERENCE_HARNESS"] = str(HARNESS)
    return env


def run_tests(extra=(), capture: bool = False) -> subprocess.CompletedProcess:
    cmd = [sys.executable, "-m", "pytest", "-p", "reference_harness_plugin", "-q",
           "tests/test_attention_decode.py", "tests/test_extreme_decode.py"]
    for item in DESELECT:
        cmd += ["--deselect", item]
    env = _env()
    env["ADB_REFERENCE_CAPABILITY_GATE"] = "1"
    return subprocess.run(cmd + list(extra), cwd=HARNESS, env=env, text=True, capture_output=capture)


def run_benchmark(extra=(), capture: bool = False) -> subprocess.CompletedProcess:
    cmd = [sys.executable, str(HERE / "reference_harness_plugin.py"), "benchmarks/bench_attention_decode.py", *extra]
    return subprocess.run(cmd, cwd=HARNESS, env=_env(), text=True, capture_output=capture)


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("what", choices=("prepare", "tests", "benchmark"))
    parser.add_argument("--reference-root")
    args, rest = parser.parse_known_args()
    if args.what == "prepare":
        if not args.reference_root:
            parser.error("prepare needs --reference-root")
        print(prepare(args.reference_root))
        return 0
    if not ready():
        print(f"{HARNESS} is not prepared (run: prepare --reference-root <checkout>)", file=sys.stderr)
        return 2
    result = run_tests(rest) if args.what == "tests" else run_benchmark(rest)
    return result.returncode


if __name__ == "__main__":
    raise SystemExit(main())
