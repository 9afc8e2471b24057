"""The allocation-free scan entry point (tkmc_scan_i32_noalloc).

Some callers cannot allocate device memory -- an in-situ hook running
inside a simulation's time step, on a GPU whose memory the simulation has
reserved, where cudaMalloc would fail or synchronise the device.  For them
the library keeps the scan's scratch in a static device array.  This checks,
through the C ABI, that two calls in a row give exactly what the
workspace-taking tkmc_scan_i32 gives and exactly the int32 prefix sums
computed on the host with numpy (int64 cumsum wrapped to int32, as the
reference's int32 fields wrap; integer results: bit-exact), and that sizes
beyond the array's limit are refused.  This file is collected last so that a
failure here leaves every other test already run.
"""

import ctypes

import numpy as np
import pytest
import torch

from tack_b200 import _lib

pytestmark = pytest.mark.gpu


def _scan_with_workspace(lib, x, inclusive):
    out = torch.empty_like(x)
    nb = lib.tkmc_scan_workspace_bytes(x.numel())
    ws = torch.empty(nb, dtype=torch.uint8, device=x.device)
    tot = ctypes.c_int64(0)
    _lib.check(lib.tkmc_scan_i32(x.data_ptr(), out.data_ptr(), x.numel(), inclusive,
                                 ws.data_ptr(), nb, ctypes.byref(tot),
                                 torch.cuda.current_stream().cuda_stream), "tkmc_scan_i32")
    return out, tot.value


def _scan_noalloc(lib, x, inclusive, want_total=True):
    out = torch.full_like(x, -1)
    tot = ctypes.c_int64(0)
    _lib.check(lib.tkmc_scan_i32_noalloc(x.data_ptr(), out.data_ptr(), x.numel(), inclusive,
                                         ctypes.byref(tot) if want_total else None,
                                         torch.cuda.current_stream().cuda_stream),
               "tkmc_scan_i32_noalloc")
    return out, tot.value


def _scan_host(a, inclusive):
    """Exact prefix sums on the host: int64 cumsum, stored as wrapped int32."""
    c = np.cumsum(a.astype(np.int64))
    ex = c if inclusive else np.concatenate([[0], c[:-1]])
    return ex.astype(np.int32), int(c[-1])


def test_noalloc_scan_matches_workspace_scan_on_consecutive_calls():
    lib = _lib.load()
    torch.cuda.set_device(0)
    rng = np.random.default_rng(2024)
    # Two calls in a row: the second starts from whatever the first left in
    # the shared static scratch.
    cases = [(3_000_017, 0, (-40, 900)), (70_001, 1, (0, 7))]
    for n, inclusive, (lo, hi) in cases:
        a = rng.integers(lo, hi, n).astype(np.int32)
        x = torch.from_numpy(a).cuda()
        ref, ref_total = _scan_with_workspace(lib, x, inclusive)
        got, got_total = _scan_noalloc(lib, x, inclusive)
        host, host_total = _scan_host(a, inclusive)
        assert got_total == ref_total == host_total
        assert torch.equal(got, ref)
        assert np.array_equal(got.cpu().numpy(), host)


def test_noalloc_scan_wraps_int32_and_runs_without_total():
    """Values whose running sum passes INT32_MAX wrap exactly as int32 fields
    do, the total stays exact in int64, and a call without a total pointer
    still returns the same prefix sums (it checks the look-back error word
    itself)."""
    lib = _lib.load()
    torch.cuda.set_device(0)
    a = np.full(1_200_000, 2_000, np.int32)  # running sum reaches 2.4e9
    x = torch.from_numpy(a).cuda()
    host, host_total = _scan_host(a, 0)
    got, got_total = _scan_noalloc(lib, x, 0)
    assert got_total == host_total == 2_400_000_000
    assert np.array_equal(got.cpu().numpy(), host)
    got2, _ = _scan_noalloc(lib, x, 1, want_total=False)
    assert np.array_equal(got2.cpu().numpy(), _scan_host(a, 1)[0])


def test_noalloc_scan_refuses_sizes_beyond_its_limit():
    lib = _lib.load()
    torch.cuda.set_device(0)
    x = torch.zeros(4, dtype=torch.int32, device="cuda")
    rc = lib.tkmc_scan_i32_noalloc(x.data_ptr(), x.data_ptr(), (1 << 26) + 1, 0, None,
                                   torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.TKMC_ERR_INVALID_ARG
    assert b"static scratch limit" in lib.tkmc_last_error()
