"""Prefix sums on int32 fields (single-pass decoupled look-back on sm_100a).

Drop-in for packages/tack-core/src/tack/algorithms/scan.py:81-123:
``exclusive_scan(input_field, output_field, n)`` and
``inclusive_scan(input_field, output_field, n)`` write int32 prefix sums and
return the total.  The reference runs ~2*log2(n)+3 synchronised launches;
this is one launch.  Sums are carried in int64: the stored int32 values wrap
exactly as the reference's int32 arithmetic does, and the returned total is
the exact int64 sum.
"""

from .. import _lib
from ..field import device_tensor, i32
from ..runtime import current_device, current_stream, workspace


def _scan(input_field, output_field, n, inclusive):
    src = device_tensor(input_field, i32)
    dst = device_tensor(output_field, i32)
    n = int(n)
    if n < 0 or n > src.numel() or n > dst.numel():
        raise ValueError(f"scan of {n} values over fields of {src.numel()} / {dst.numel()}")
    lib = _lib.load()
    dev = current_device()
    ws = workspace("scan", lib.tkmc_scan_workspace_bytes(n), dev)
    import ctypes
    total = ctypes.c_int64(0)
    _lib.check(lib.tkmc_scan_i32(src.data_ptr(), dst.data_ptr(), n, 1 if inclusive else 0,
                                 ws.data_ptr(), ws.numel(), ctypes.byref(total),
                                 current_stream(dev)), "tkmc_scan_i32")
    return int(total.value)


def exclusive_scan(input_field, output_field, n):
    """output[i] = sum(input[0..i-1]), output[0] = 0; returns the total."""
    return _scan(input_field, output_field, n, False)


def inclusive_scan(input_field, output_field, n):
    """output[i] = sum(input[0..i]); returns the total."""
    return _scan(input_field, output_field, n, True)
