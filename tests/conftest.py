import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def golden_manifest():
    import json
    with open(os.path.join(REPO, "tests", "golden", "manifest.json")) as f:
        return json.load(f)


def pytest_sessionfinish(session, exitstatus):
    """With the bounds-checked library (FFTS_LIBRARY=checked), fail the session if
    any kernel index check failed during the tests, and write the records (JSON)
    to the file named by FFTS_BOUNDS_REPORT when it is set."""
    if os.environ.get("FFTS_LIBRARY", "") != "checked" or not cuda_ok():
        return
    import json
    from fftsparse_b200 import _lib
    if _lib._lib is None:  # no test loaded the library
        records, enabled = [], None
    else:
        import torch
        torch.cuda.synchronize()
        records = _lib.bounds_report(clear=True)
        enabled = int(_lib._lib.ffts_bounds_check_enabled())
    out = os.environ.get("FFTS_BOUNDS_REPORT")
    if out:
        with open(out, "w") as f:
            json.dump({"library": _lib.LIB_PATH, "checks_compiled": enabled, "records": records}, f)
    if records:
        print(f"\nbounds-checked build: failed index checks {records}")
        session.exitstatus = 1
