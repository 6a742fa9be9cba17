"""C-ABI checks that need no GPU: the library loads, exports every symbol the
public header declares with the expected signature, and rejects bad arguments
before touching the device."""
import ctypes
import os
import re

import pytest

from fftsparse_b200 import _lib
from fftsparse_b200.params import CMaskParams, derive_mask_params

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "fftsparse_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ffts_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    assert set(names) == set(_lib.EXPORTS), (names, sorted(_lib.EXPORTS))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} missing from {_lib.LIB_PATH}"


def test_version_and_error_string_without_gpu():
    lib = _lib.load()
    assert lib.ffts_version() >= 100
    assert isinstance(lib.ffts_last_error_string(), bytes)


def test_workspace_query_is_host_only():
    lib = _lib.load()
    assert lib.ffts_mask_workspace_bytes(1, 32, 1024, 128) > 0
    assert lib.ffts_mask_workspace_bytes(0, 32, 1024, 128) == 0


def test_params_struct_layout_matches_header():
    # ffts_mask_params: 13 scalars, 64 sampled lags, 9 trailing scalars (4 bytes each)
    assert ctypes.sizeof(CMaskParams) == 4 * (13 + 64 + 9)


def test_params_derivation_efficiency_settings():
    p = derive_mask_params(131072, sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02,
                           correlation_selection_mode="topk", correlation_topk_ratio=0.05,
                           column_topk_ratio=0.2)
    # values quoted for N = 1024 from my_attn_v7.py:537-540, 583-594, 626-634
    assert (p.n_blocks, p.keep_sink, p.keep_recent, p.local_window) == (1024, 10, 1, 10)
    assert p.remote_start == 11 and p.sink_tau_raw == 1024 - 10 - 5
    assert (p.col_start, p.col_end, p.col_topk) == (102, 820, 50)
    assert len(p.diag_taus) == 64 and p.diag_taus[0] == 11
    assert p.last_topk == 128


@pytest.mark.parametrize("L,ratio,want", [
    # N, keep_sink, keep_recent, local_window, remote_start, FFT cut, columns, column top-k,
    # stripe samples, last-row top-k (BASELINE configs 1 and 2 with the efficiency-script ratios)
    (8192, 0.1, (64, 1, 1, 1, 2, 58, 6, 52, 9, 5, 64)),
    (32768, 0.05, (256, 2, 1, 2, 3, 249, 25, 205, 25, 19, 128)),
    (131072, 0.05, (1024, 10, 1, 10, 11, 1009, 102, 820, 50, 64, 128)),
])
def test_params_derivation_baseline_configs(L, ratio, want):
    p = derive_mask_params(L, sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02,
                           correlation_selection_mode="topk", correlation_topk_ratio=ratio,
                           qk_topk_ratio=ratio, column_topk_ratio=0.2, diag_sample_ratio=0.15,
                           min_diag_samples=5, max_diag_samples=64)
    got = (p.n_blocks, p.keep_sink, p.keep_recent, p.local_window, p.remote_start, p.sink_tau_raw,
           p.col_start, p.col_end, p.col_topk, len(p.diag_taus), p.last_topk)
    assert got == want


def test_unknown_selection_mode_raises_value_error():
    with pytest.raises(ValueError):
        derive_mask_params(8192, correlation_selection_mode="bogus")


def test_remote_start_beyond_blocks_raises():
    with pytest.raises(ValueError):
        derive_mask_params(1280, recent_ratio=1.0)


def test_checked_library_exports_the_same_symbols():
    """The bounds-checked build exports every symbol of the header and says so."""
    import ctypes
    from fftsparse_b200 import _lib
    assert os.path.exists(_lib.LIB_CHECKED), "build the checked library: python -m fftsparse_b200.build"
    checked = ctypes.CDLL(_lib.LIB_CHECKED)
    for name in _lib.EXPORTS:
        assert hasattr(checked, name), f"{name} missing from {_lib.LIB_CHECKED}"
    checked.ffts_bounds_check_enabled.restype = ctypes.c_int32
    assert checked.ffts_bounds_check_enabled() == 1
    normal = ctypes.CDLL(_lib.LIB_NORMAL)
    normal.ffts_bounds_check_enabled.restype = ctypes.c_int32
    assert normal.ffts_bounds_check_enabled() == 0
    # the normal build has no records and touches no device to say so
    normal.ffts_bounds_report.restype = ctypes.c_int32
    normal.ffts_bounds_report.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32]
    assert normal.ffts_bounds_report(None, 0, 1) == 0
