"""The reference's own test files, unmodified, against this package.

baseline/reference_harness.py runs the reference's
tests/test_attention_decode.py and tests/test_extreme_decode.py in a
subprocess where ``attention_decode`` is this package and
``attention_decode.reference`` is the reference's own FP32 oracle, with the
two documented differences only: the capability gate reports (12, 0) on a
10.x device, and the case that requires a GQA group of 8 to be rejected is
deselected (this build supports it).  The harness files are copied by
``__graft_entry__.build()`` where a reference checkout is present; without
them this test is skipped.
"""

from __future__ import annotations

import os
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "baseline"))

import reference_harness  # noqa: E402


def test_reference_test_files_pass_unmodified(cuda_device):
    if not reference_harness.ready():
        pytest.skip("reference harness not prepared (build() copies it where a reference checkout exists)")
    result = reference_harness.run_tests(["-p", "no:cacheprovider"], capture=True)
    tail = result.stdout[-4000:] + result.stderr[-2000:]
    assert result.returncode == 0, tail
    summary = result.stdout.strip().splitlines()[-1]
    assert " passed" in summary and "failed" not in summary and "skipped" not in summary, summary
    assert "1 deselected" in summary, summary
