"""Import set-up for running the reference's own test and benchmark files
against this package (see baseline/reference_harness.py).

As a pytest plugin (``-p reference_harness_plugin``) or as a launcher
(``python reference_harness_plugin.py <script> [args]``) it:
  * imports this package as ``attention_decode`` and registers the
    reference's own reference.py (copied into the harness directory named by
    ADB_REFERENCE_HARNESS) as ``attention_decode.reference``;
  * with ADB_REFERENCE_CAPABILITY_GATE=1, makes
    torch.cuda.get_device_capability() report (12, 0) on a compute-capability
    10.x device, which is the reference fixtures' gate
    (tests/test_attention_decode.py:36-42, tests/test_extreme_decode.py:16-19).
"""

from __future__ import annotations

import importlib.util
import os
import runpy
import sys
from pathlib import Path


def _install() -> None:
    harness = Path(os.environ["ADB_REFERENCE_HARNESS"])
    import torch

    import attention_decode

    if "attention_decode.reference" not in sys.modules:
        spec = importlib.util.spec_from_file_location("attention_decode.reference", harness / "reference.py")
        module = importlib.util.module_from_spec(spec)
        sys.modules["attention_decode.reference"] = module
        spec.loader.exec_module(module)
        attention_decode.reference = module
    if os.environ.get("ADB_REFERENCE_CAPABILITY_GATE") == "1":
        real = torch.cuda.get_device_capability

        def gate(device=None):
            major, minor = real(device)
            return (12, 0) if major == 10 else (major, minor)

        torch.cuda.get_device_capability = gate


_install()

if __name__ == "__main__":
    script = sys.argv[1]
    sys.argv = sys.argv[1:]
    runpy.run_path(script, run_name="__main__")
