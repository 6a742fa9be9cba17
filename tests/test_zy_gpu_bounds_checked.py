"""The GPU parity tests, run again on the bounds-checked library.

libfftsparse_b200_checked.so is the same CUDA sources compiled with
-DFFTS_BOUNDS_CHECK: each index that comes from data or from a ragged edge
(mask words, tile cursors, sampled lags, selected columns, output rows, key
rows, CSR positions) is tested against its extent, and a failure is counted on
the device and the access skipped instead of faulting.  This test runs every
other single-GPU test in a child process with FFTS_LIBRARY=checked, so the same
odd shapes, golden fixtures and edge cases pass through the checked kernels;
it passes when the child's tests pass and no check failed
(ffts_bounds_report, collected by tests/conftest.py at the child's session end).
"""
import json
import os
import subprocess
import sys

import pytest

from conftest import REPO, cuda_ok

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not cuda_ok(), reason="needs a GPU")
def test_gpu_suite_passes_on_the_bounds_checked_library(tmp_path):
    from fftsparse_b200 import _lib
    assert os.path.exists(_lib.LIB_CHECKED), "build the checked library: python -m fftsparse_b200.build"
    report = tmp_path / "bounds.json"
    env = dict(os.environ, FFTS_LIBRARY="checked", FFTS_BOUNDS_REPORT=str(report))
    cmd = [sys.executable, "-m", "pytest", os.path.join(REPO, "tests"), "-m", "gpu", "-x", "-q",
           "-p", "no:cacheprovider",
           "--ignore", os.path.join(REPO, "tests", os.path.basename(__file__)),
           "--ignore", os.path.join(REPO, "tests", "test_gpu_peer.py")]  # needs two GPUs
    res = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=1500)
    tail = (res.stdout + res.stderr)[-4000:]
    assert res.returncode == 0, f"GPU tests on the checked library failed:\n{tail}"
    assert report.exists(), f"the child session wrote no bounds report:\n{tail}"
    rep = json.loads(report.read_text())
    assert rep["checks_compiled"] == 1 and rep["library"] == _lib.LIB_CHECKED, rep
    assert rep["records"] == [], f"failed index checks: {rep['records']}"
