"""ctypes binding of libfftsparse_b200.so (the C ABI in include/fftsparse_b200.h).

The library is required: importing the operators without it raises, and there
is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NORMAL = os.path.join(HERE, "libfftsparse_b200.so")
# The bounds-checked build (every data-dependent kernel index tested, failures
# recorded and skipped; slower) is loaded instead when FFTS_LIBRARY=checked.
LIB_CHECKED = os.path.join(HERE, "libfftsparse_b200_checked.so")
LIB_PATH = LIB_CHECKED if os.environ.get("FFTS_LIBRARY", "") == "checked" else LIB_NORMAL

FFTS_OK = 0
FFTS_E_INVALID = -1
FFTS_E_UNSUPPORTED = -2
FFTS_E_CUDA = -3
FFTS_E_WORKSPACE = -4
FFTS_E_DEVICE = -5

DTYPE_F32 = 0
DTYPE_BF16 = 1

# (name, restype, argtypes) of every export declared in include/fftsparse_b200.h
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
EXPORTS = {
    "ffts_version": (_I32, []),
    "ffts_last_error_string": (ctypes.c_char_p, []),
    "ffts_init": (_I32, [_I32]),
    "ffts_pool": (_I32, [_P, _I32, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _P, _P]),
    "ffts_mask_workspace_bytes": (_I64, [_I64, _I64, _I64, _I64]),
    "ffts_block_mask": (_I32, [_P, _P, _I32, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P,
                               _I64, _P]),
    "ffts_block_mask_noalloc": (_I32, [_P, _P, _I32, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P,
                                       _P]),
    "ffts_unpack_mask": (_I32, [_P, _I64, _I64, _I64, _P, _P]),
    "ffts_mask_row_ptr": (_I32, [_P, _I64, _P, _P]),
    "ffts_mask_col_idx": (_I32, [_P, _I64, _I64, _P, _P, _I64, _P, _P]),
    "ffts_rope_pool": (_I32, [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I32,
                              _P, _P, _P, _P, _P, _P]),
    "ffts_qkv_rope_pool": (_I32, [_P, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P, _I64, _I64, _I64, _P, _P, _I64,
                                  _I32, _P, _P, _P, _P, _P, _P, _I64, _P, _I64, _P, _P]),
    "ffts_qkv_workspace_bytes": (_I64, [_I64]),
    "ffts_decode_workspace_bytes": (_I64, [_I64, _I64, _I64, _I64]),
    "ffts_decode_attn": (_I32, [_P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P,
                                _I64, _I64, _P, _I32, _I64, _P]),
    "ffts_sparse_attn_fwd": (_I32, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _I32,
                                    _I32, _P, _P, _P, _P]),
    "ffts_sparse_attn_fwd_rows": (_I32, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _I32,
                                         _I32, _I64, _I64, _P, _P, _P, _P]),
    "ffts_sparse_attn_fwd_push": (_I32, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _I32,
                                         _I32, _I64, _I64, _P, _P, _P, _I32, _P, _P]),
    "ffts_ipc_handle": (_I32, [_P, _P, _P]),
    "ffts_ipc_open": (_I32, [_P, _I64, _P]),
    "ffts_ipc_close": (_I32, [_P, _I64]),
    "ffts_copy_rows": (_I32, [_P, _P, _I32, _P, _I64, _I64, _I64, _P]),
    "ffts_copy_2d": (_I32, [_P, _I64, _P, _I64, _I64, _I64, _P]),
    "ffts_signal": (_I32, [_P, _P, _I32, _I32]),
    "ffts_wait_flags": (_I32, [_P, _I32, _I32, _P, _P]),
    "ffts_bounds_check_enabled": (_I32, []),
    "ffts_bounds_report": (_I32, [_P, _I32, _I32]),
}

_lib = None


class FFTSparseError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{message} [ffts code {code}]")
        self.code = code


def load(path: str = LIB_PATH):
    """Load (once) and return the ctypes handle; raises if the library is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{os.path.basename(path)} not found at {path}; build it with "
            "`python -m fftsparse_b200.build` (nvcc, sm_100a). There is no CPU fallback.")
    lib = ctypes.CDLL(path)
    for name, (res, args) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class BoundsRecord(ctypes.Structure):
    """ffts_bounds_record of include/fftsparse_b200.h."""
    _fields_ = [("file", ctypes.c_char * 48), ("line", ctypes.c_int32), ("count", ctypes.c_uint32),
                ("block", ctypes.c_int64)]


def bounds_report(clear: bool = True, max_records: int = 32):
    """Failed index checks of the bounds-checked build on the current device, one
    dict per source file (file, line of the first failure, count, block); always
    empty with the normal build."""
    lib = load()
    recs = (BoundsRecord * max_records)()
    n = lib.ffts_bounds_report(recs, max_records, int(bool(clear)))
    if n < 0:
        check(n)
    return [{"file": r.file.decode(), "line": r.line, "count": r.count, "block": r.block}
            for r in recs[:min(n, max_records)]]


def check(rc: int) -> None:
    if rc == FFTS_OK:
        return
    msg = load().ffts_last_error_string().decode(errors="replace")
    if rc == FFTS_E_INVALID:
        raise ValueError(msg)
    if rc == FFTS_E_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise FFTSparseError(rc, msg)


def i64_array(values):
    arr = (ctypes.c_int64 * len(values))(*[int(v) for v in values])
    return arr
