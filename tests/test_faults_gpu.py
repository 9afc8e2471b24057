"""Bounded device-side waits end in an error status, never a hang.

The decoupled look-back spins on predecessor tiles' status flags.  A test
hook makes one tile skip publishing its status, so its successors' waits can
only end by the time limit (set short here); the call must return
TKMC_ERR_DEVICE_TIMEOUT, and the context must stay usable.  Nothing faults,
traps or hangs the GPU.
"""

import numpy as np
import pytest
import torch

from conftest import load_fe_case
from fe_helpers import capi_fe, f32arr, stream
from tack_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.fixture
def short_wait():
    lib = _lib.load()
    lib.tkmc_set_wait_limit_ns(20_000_000)  # 20 ms
    yield lib
    lib.tkmc_set_wait_limit_ns(0)
    lib.tkmc_test_skip_publish(-1)


def test_fe_scan_wait_expires_with_status(tack, short_wait):
    lib = short_wait
    c = load_fe_case("gyroid48")  # 48*48 node rows -> 3 scan tiles of 1024 rows
    nx, ny, nz = c["grid_tuple"][:3]
    v = torch.from_numpy(c["values"]).cuda()
    nb = lib.tkmc_fe_workspace_bytes(nx, ny, nz, 1)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    counts = np.zeros(4, np.int64)
    lib.tkmc_test_skip_publish(1)
    rc = lib.tkmc_fe_count(v.data_ptr(), nx, ny, nz, 0, f32arr([0.0]), 1, None, ws.data_ptr(), nb,
                           counts.ctypes.data, stream())
    assert rc == _lib.TKMC_ERR_DEVICE_TIMEOUT
    assert b"wait expired" in lib.tkmc_last_error()
    # The context is intact: the next call succeeds and matches the reference.
    got = capi_fe(c["values"], c["grid_tuple"], [0.0])
    np.testing.assert_array_equal(got["conn"], c["conn"])


def test_scan_wait_expires_with_status(tack, short_wait):
    lib = short_wait
    n = 5 * 4096 + 17
    a = torch.ones(n, dtype=torch.int32, device="cuda")
    out = torch.empty_like(a)
    nb = lib.tkmc_scan_workspace_bytes(n)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    import ctypes
    tot = ctypes.c_int64(0)
    lib.tkmc_test_skip_publish(2)
    rc = lib.tkmc_scan_i32(a.data_ptr(), out.data_ptr(), n, 0, ws.data_ptr(), nb,
                           ctypes.byref(tot), stream())
    assert rc == _lib.TKMC_ERR_DEVICE_TIMEOUT
    rc = lib.tkmc_scan_i32(a.data_ptr(), out.data_ptr(), n, 0, ws.data_ptr(), nb,
                           ctypes.byref(tot), stream())
    assert rc == 0 and tot.value == n
    assert torch.equal(out.cpu(), torch.arange(n, dtype=torch.int32))



def test_exchange_wait_expires_with_status(tack, short_wait):
    """A peer that never runs its totals exchange: rank 0's wait for the
    peer's flag (a flag nothing sets) ends by the time limit, the status is
    read back by tkmc_fe_check, and the context stays usable.  Both ranks'
    exchanges live in this process; only rank 0 launches."""
    import ctypes
    lib = short_wait
    c = load_fe_case("gyroid48")
    nx, ny, nz = c["grid_tuple"][:3]
    v = torch.from_numpy(c["values"]).cuda()
    nb = lib.tkmc_fe_workspace_bytes(nx, ny, nz, 1)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    counts = np.zeros(4, np.int64)
    assert lib.tkmc_fe_count(v.data_ptr(), nx, ny, nz, 0, f32arr([0.0]), 1, None, ws.data_ptr(),
                             nb, counts.ctypes.data, stream()) == 0
    hb = lib.tkmc_exchange_handle_bytes()
    ex = [ctypes.c_void_p(), ctypes.c_void_p()]
    handles = [ctypes.create_string_buffer(hb) for _ in ex]
    for r in range(2):
        assert lib.tkmc_exchange_create(2, r, 1, ctypes.byref(ex[r]), handles[r]) == 0
    try:
        members = (ctypes.c_void_p * 2)(ex[0].value, ex[1].value)
        assert lib.tkmc_exchange_connect_local(ex[0], members) == 0
        bad = (ctypes.c_void_p * 2)(ex[1].value, ex[0].value)  # wrong rank order
        assert lib.tkmc_exchange_connect_local(ex[0], bad) == _lib.TKMC_ERR_INVALID_ARG
        bases = torch.zeros(7, dtype=torch.int64, device="cuda")
        assert lib.tkmc_exchange_plan(ex[0], nx, ny, nz, 0, ws.data_ptr(), nb, 0,
                                      bases.data_ptr(), stream()) == 0
        rc = lib.tkmc_fe_check(nx, ny, nz, 1, ws.data_ptr(), nb, stream())
        assert rc == _lib.TKMC_ERR_DEVICE_TIMEOUT
        assert b"wait expired" in lib.tkmc_last_error()
    finally:
        torch.cuda.synchronize()
        for x in ex:
            lib.tkmc_exchange_destroy(x)
    got = capi_fe(c["values"], c["grid_tuple"], [0.0])
    np.testing.assert_array_equal(got["conn"], c["conn"])


def test_scan_timeout_reported_without_total(tack, short_wait):
    """With total == NULL the scan still reads its look-back error word back,
    so an expired wait is reported."""
    lib = short_wait
    n = 5 * 4096 + 17
    a = torch.ones(n, dtype=torch.int32, device="cuda")
    out = torch.empty_like(a)
    nb = lib.tkmc_scan_workspace_bytes(n)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    lib.tkmc_test_skip_publish(3)
    rc = lib.tkmc_scan_i32(a.data_ptr(), out.data_ptr(), n, 0, ws.data_ptr(), nb, None, stream())
    assert rc == _lib.TKMC_ERR_DEVICE_TIMEOUT
    assert lib.tkmc_scan_i32(a.data_ptr(), out.data_ptr(), n, 1, ws.data_ptr(), nb, None,
                             stream()) == 0
    assert torch.equal(out.cpu(), torch.arange(1, n + 1, dtype=torch.int32))


@pytest.mark.parametrize("shape", ["unaligned", "aligned"])
def test_device_plan_refuses_point_ids_beyond_int32(tack, shape):
    """Device-side planning from gathered totals whose global point count
    exceeds INT32_MAX: the plan marks the bases, every emit kernel then writes
    nothing and records TKMC_ERR_OVERFLOW, which tkmc_fe_check returns.
    The totals of the other rank are faked (2^31 points); this rank's own
    slab is a real volume (rows of 49 nodes: the word-granular emit; rows of
    64 nodes: the unit-driven emit)."""
    import ctypes
    from tack_b200 import workloads
    lib = _lib.load()
    if shape == "unaligned":
        c = load_fe_case("gyroid48")
        nx, ny, nz = c["grid_tuple"][:3]
        v = torch.from_numpy(c["values"]).cuda()
        iso = 0.0
    else:
        nx = ny = nz = 63
        v = workloads.generate("sphere")
        iso = 0.0
    nb = lib.tkmc_fe_workspace_bytes(nx, ny, nz, 1)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    counts = np.zeros(4, np.int64)
    _lib.check(lib.tkmc_fe_count(v.data_ptr(), nx, ny, nz, 0, f32arr([iso]), 1, None,
                                 ws.data_ptr(), nb, counts.ctypes.data, stream()), "count")
    assert counts[:3].sum() > 0 and counts[3] > 0
    # Rank 0 (this slab) and a faked rank 1 whose x section alone holds 2^31 points.
    allc = torch.tensor(np.concatenate([counts, [1 << 31, 0, 0, 0]]), dtype=torch.int64,
                        device="cuda")
    bases = torch.zeros(7, dtype=torch.int64, device="cuda")
    _lib.check(lib.tkmc_fe_plan(allc.data_ptr(), 2, 0, 1, 0, bases.data_ptr(), stream()), "plan")
    P, T = int(counts[:3].sum()), int(counts[3])
    pts = torch.full((P * 3,), 7.0, dtype=torch.float32, device="cuda")
    conn = torch.full((T * 3,), -7, dtype=torch.int32, device="cuda")
    geom = f32arr([0.0, 0.0, 0.0, 1.0, 1.0, 1.0])
    _lib.check(lib.tkmc_fe_emit_dev(v.data_ptr(), nx, ny, nz, 0, 0, geom, f32arr([iso]), 1, None,
                                    ws.data_ptr(), nb, bases.data_ptr(), pts.data_ptr(), P,
                                    conn.data_ptr(), T, stream()), "emit_dev")
    rc = lib.tkmc_fe_check(nx, ny, nz, 1, ws.data_ptr(), nb, stream())
    assert rc == _lib.TKMC_ERR_OVERFLOW
    assert b"int32 point ids" in lib.tkmc_last_error()
    assert bool((pts == 7.0).all()) and bool((conn == -7).all())
    # Totals that fit (rank 1 with triangles only, so this rank's point ids
    # are those of the volume alone): the same calls emit the single-volume
    # connectivity.
    allc_ok = torch.tensor(np.concatenate([counts, [0, 0, 0, 5]]), dtype=torch.int64,
                           device="cuda")
    _lib.check(lib.tkmc_fe_count(v.data_ptr(), nx, ny, nz, 0, f32arr([iso]), 1, None,
                                 ws.data_ptr(), nb, counts.ctypes.data, stream()), "count")
    _lib.check(lib.tkmc_fe_plan(allc_ok.data_ptr(), 2, 0, 1, 0, bases.data_ptr(), stream()),
               "plan")
    _lib.check(lib.tkmc_fe_emit_dev(v.data_ptr(), nx, ny, nz, 0, 0, geom, f32arr([iso]), 1, None,
                                    ws.data_ptr(), nb, bases.data_ptr(), pts.data_ptr(), P,
                                    conn.data_ptr(), T, stream()), "emit_dev")
    _lib.check(lib.tkmc_fe_check(nx, ny, nz, 1, ws.data_ptr(), nb, stream()), "check")
    got = capi_fe(v, (nx, ny, nz, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0), [iso])
    np.testing.assert_array_equal(conn.cpu().numpy().reshape(-1, 3), got["conn"])
