"""Dynamic load balancing (work stealing) forced on at sizes where the
default policy leaves it off, checked against the CPU oracle.

Stealing turns one pair's tiles into more segments than its static owners
(thief segments found by tag, owner segments emptied by thieves, the last
contribution merging from its own shared-memory state), so every case runs
with it on in a child process: the knobs are read once per process.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("claim_divisor", ("2", "4"))
def test_forced_stealing_matches_oracle(claim_divisor, device):
    env = dict(os.environ, ADB_MAX_STEALS="16", ADB_CLAIM_DIVISOR=claim_divisor, ADB_DETERMINISTIC="0")
    proc = subprocess.run(
        [sys.executable, os.path.join(HERE, "forced_steal_child.py")],
        env=env, capture_output=True, text=True, timeout=600,
    )
    assert proc.returncode == 0, proc.stderr[-4000:]
    results = [json.loads(line) for line in proc.stdout.splitlines() if line.startswith("{")]
    assert len(results) == 7, proc.stdout
    for r in results:
        assert r["finite"], r
        assert r["excess"] <= 0.0, r
        assert r["partial_excess"] <= 0.0, r
        assert r["error_flag"] == 0, r
