"""The bounds-checked build (libturbocider_cuda_checked.so, -DTC_BOUNDS_CHECK):
the substitute for compute-sanitizer, which this GPU pool does not offer.
Every output store, weight-chunk address, decode target offset and split-K
share read is checked against the extent the host passed; an index outside
sets STATUS_BOUNDS and the access is skipped (or a read clamped) instead of
faulting.  The workload (tests/checked_workload.py) runs every kernel family
on ragged shapes in a fresh process with that library loaded and requires a
clear status after every call."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def test_checked_build_sees_no_out_of_bounds_access():
    lib = HERE.parent / "turbocider_b200" / "libturbocider_cuda_checked.so"
    if not lib.exists():
        pytest.fail("the bounds-checked library was not built (python -m turbocider_b200.build)")
    env = dict(os.environ, TURBOCIDER_CHECKED="1")
    r = subprocess.run([sys.executable, str(HERE / "checked_workload.py")], env=env, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "no bounds violation" in r.stdout
