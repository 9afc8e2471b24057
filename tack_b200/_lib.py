"""ctypes binding of libtackmc.so (declared in include/tackmc.h).

The library is the only compute path: there is no CPU or PyTorch fallback.
If it is missing or cannot be loaded, every entry point raises.
"""

import ctypes
import os
import threading

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "libtackmc.so")

TKMC_OK = 0
TKMC_ERR_INVALID_ARG = 1
TKMC_ERR_WORKSPACE = 2
TKMC_ERR_OVERFLOW = 3
TKMC_ERR_DEVICE_TIMEOUT = 4
TKMC_ERR_CUDA = 5
TKMC_ERR_CAPACITY = 6
MAX_ISO = 8

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/tackmc.h
SIGNATURES = {
    "tkmc_version": (_I, []),
    "tkmc_last_error": (ctypes.c_char_p, []),
    "tkmc_launch_count": (ctypes.c_uint64, []),
    "tkmc_mc_tables": (_I, [_P, _P, _P]),
    "tkmc_reduce_workspace_bytes": (_SZ, [_I64]),
    "tkmc_reduce_f32": (_I, [_P, _I64, _P, _SZ, _P, _P]),
    "tkmc_scan_workspace_bytes": (_SZ, [_I64]),
    "tkmc_scan_i32": (_I, [_P, _P, _I64, _I, _P, _SZ, _P, _P]),
    "tkmc_scan_i32_noalloc": (_I, [_P, _P, _I64, _I, _P, _P]),
    "tkmc_normals_workspace_bytes": (_SZ, [_I64]),
    "tkmc_compute_normals": (_I, [_P, _P, _I64, _I64, _P, _SZ, _P, _P]),
    "tkmc_fe_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I]),
    "tkmc_fe_emit_dev": (_I, [_P, _I64, _I64, _I64, _I, _I64, _P, _P, _I, _P, _P, _SZ, _P, _P,
                              _I64, _P, _I64, _P]),
    "tkmc_fe_copy_counts": (_I, [_I64, _I64, _I64, _I, _P, _SZ, _P, _P]),
    "tkmc_fe_copy_status": (_I, [_I64, _I64, _I64, _I, _P, _SZ, _P, _P]),
    "tkmc_fe_batch_stride": (_SZ, [_I64, _I64, _I64, _I]),
    "tkmc_fe_count_batch": (_I, [_P, _I64, _I64, _I64, _I64, _P, _I, _P, _P, _SZ, _P, _P, _P]),
    "tkmc_fe_emit_batch": (_I, [_P, _I64, _I64, _I64, _I64, _P, _P, _I, _P, _P, _SZ, _P, _P,
                                _I64, _P, _I64, _P, _P]),
    "tkmc_exchange_handle_bytes": (_SZ, []),
    "tkmc_exchange_create": (_I, [_I, _I, _I, _P, _P]),
    "tkmc_exchange_connect": (_I, [_P, _P]),
    "tkmc_exchange_connect_local": (_I, [_P, _P]),
    "tkmc_exchange_plan": (_I, [_P, _I64, _I64, _I64, _I, _P, _SZ, _I, _P, _P]),
    "tkmc_exchange_destroy": (_I, [_P]),
    "tkmc_exchange_plan_counts": (_I, [_P, _I64, _I64, _I64, _I, _P, _SZ, _I, _P, _P]),
    "tkmc_fe_emit_soup": (_I, [_P, _I64, _I64, _I64, _P, _P, _I, _P, _P, _SZ, _P, _P, _P, _P,
                               _I64, _P]),
    "tkmc_fe_plan": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "tkmc_fe_clear_capacity_error": (_I, [_I64, _I64, _I64, _I, _P, _SZ, _P]),
    "tkmc_fe_count": (_I, [_P, _I64, _I64, _I64, _I, _P, _I, _P, _P, _SZ, _P, _P]),
    "tkmc_fe_emit": (_I, [_P, _I64, _I64, _I64, _I, _I64, _P, _P, _I, _P, _P, _SZ,
                          _P, _P, _P, _P, _I64, _P, _I64, _P]),
    "tkmc_fe_check": (_I, [_I64, _I64, _I64, _I, _P, _SZ, _P]),
    "tkmc_fe_classify": (_I, [_P, _I64, _I64, _I64, _P, _I, _P, _SZ, _P]),
    "tkmc_fe_scan": (_I, [_I64, _I64, _I64, _I, _I, _P, _P, _SZ, _P]),
    "tkmc_fe_scan_part": (_I, [_I64, _I64, _I64, _I, _I, _P, _P, _SZ, _I, _P]),
    "tkmc_fe_read_counts": (_I, [_I64, _I64, _I64, _I, _P, _SZ, _P, _P]),
    "tkmc_fe_row_offsets": (_I, [_I64, _I64, _I64, _I, _I, _P, _SZ, _P, _P]),
    "tkmc_fe_run": (_I, [_P, _I64, _I64, _I64, _P, _P, _I, _P, _P, _SZ, _P, _I64, _P, _I64,
                         _P, _P]),
    "tkmc_mc_classify_cells": (_I, [_P, _I64, _I64, _I64, _F, _P, _P, _SZ, _P, _P, _P]),
    "tkmc_set_wait_limit_ns": (None, [_I64]),
    "tkmc_test_skip_publish": (None, [_I64]),
}

_lib = None
_lock = threading.Lock()


class TkmcError(RuntimeError):
    """A libtackmc call failed; ``code`` is the TKMC_ERR_* status."""

    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


def load():
    """Load libtackmc.so once; raise if it is absent (no fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"libtackmc.so not found at {LIB_PATH}; build it with "
                    "`python -m tack_b200._build` (nvcc, sm_100a). tack_b200 has no CPU "
                    "fallback.")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc, what):
    """Raise TkmcError for a non-zero status, with the library's message."""
    if rc != TKMC_OK:
        msg = load().tkmc_last_error().decode(errors="replace")
        raise TkmcError(rc, f"{what}: {msg} (status {rc})")
    return rc
