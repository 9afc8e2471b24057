"""Helpers for GPU parity tests: call libtackmc.so through its C ABI.

These drive the library exactly as a foreign caller would (ctypes, raw
device pointers, caller-owned workspace and outputs), independent of the
tack_b200 Python layer.
"""

import ctypes

import numpy as np
import torch

from tack_b200 import _lib


def f32arr(vals):
    return (ctypes.c_float * len(vals))(*vals)


def i64arr(vals):
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def stream():
    return torch.cuda.current_stream().cuda_stream


def capi_fe(values, grid, isovalues, mask=None, want_rows=False, host=True):
    """Count + emit through the C ABI; returns dict of host arrays (points
    and conn stay CUDA tensors, shaped (-1, 3), when host is False).

    values: flat f32 CUDA tensor or numpy array.  grid: (nx, ny, nz, x0, y0,
    z0, dx, dy, dz).  isovalues: list (<= 8).
    """
    lib = _lib.load()
    nx, ny, nz = grid[:3]
    v = values if isinstance(values, torch.Tensor) else torch.from_numpy(
        np.ascontiguousarray(values, np.float32)).cuda()
    m = None
    if mask is not None:
        m = mask if isinstance(mask, torch.Tensor) else torch.from_numpy(
            np.ascontiguousarray(mask, np.int32)).cuda()
    niso = len(isovalues)
    nbytes = lib.tkmc_fe_workspace_bytes(nx, ny, nz, niso)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    counts = np.zeros(4 * niso, np.int64)
    _lib.check(lib.tkmc_fe_count(v.data_ptr(), nx, ny, nz, 0, f32arr(isovalues), niso,
                                 m.data_ptr() if m is not None else None, ws.data_ptr(), nbytes,
                                 counts.ctypes.data, stream()), "tkmc_fe_count")
    rows = None
    if want_rows:
        R = (ny + 1) * (nz + 1)
        rows = []
        for q in range(niso):
            out = np.zeros(R * 4, np.int64)
            _lib.check(lib.tkmc_fe_row_offsets(nx, ny, nz, niso, q, ws.data_ptr(), nbytes,
                                               out.ctypes.data, stream()), "row_offsets")
            rows.append(out.reshape(R, 4))
    ids, tri = [], []
    P = T = 0
    for q in range(niso):
        X, Y, Z, Tq = (int(c) for c in counts[4 * q:4 * q + 4])
        ids += [P, P + X, P + X + Y]
        tri.append(T)
        P += X + Y + Z
        T += Tq
    pts = torch.full((max(P, 1) * 3,), float("nan"), dtype=torch.float32, device="cuda")
    conn = torch.full((max(T, 1) * 3,), -7, dtype=torch.int32, device="cuda")
    _lib.check(lib.tkmc_fe_emit(v.data_ptr(), nx, ny, nz, 0, 0, f32arr(grid[3:]),
                                f32arr(isovalues), niso, m.data_ptr() if m is not None else None,
                                ws.data_ptr(), nbytes, i64arr(ids), i64arr(ids), i64arr(tri),
                                pts.data_ptr(), P, conn.data_ptr(), T, stream()), "tkmc_fe_emit")
    _lib.check(lib.tkmc_fe_check(nx, ny, nz, niso, ws.data_ptr(), nbytes, stream()),
               "tkmc_fe_check")
    torch.cuda.synchronize()
    if not host:
        return {"counts": counts.reshape(niso, 4), "points": pts[:P * 3].view(-1, 3),
                "conn": conn[:T * 3].view(-1, 3), "rows": rows, "total_points": P,
                "total_tris": T}
    return {"counts": counts.reshape(niso, 4), "points": pts[:P * 3].cpu().numpy().reshape(-1, 3),
            "conn": conn[:T * 3].cpu().numpy().reshape(-1, 3), "rows": rows,
            "total_points": P, "total_tris": T}


def reference_offsets_from_rows(rows, counts, grid):
    """Convert the library's section-relative row offsets into the
    reference's _count_block arrays (xo, yo + X, zo + X + Y, cell-row tri
    offsets)."""
    nx, ny, nz = grid[:3]
    X, Y = int(counts[0]), int(counts[1])
    xo = rows[:, 0]
    yo = rows[:, 1] + X
    zo = rows[:, 2] + X + Y
    r = rows[:, 3].reshape(nz + 1, ny + 1)[:nz, :ny].reshape(-1)
    return xo, yo, zo, r


def assert_points_identical(a, b):
    """Bit-identical f32 coordinates, NaN payloads aside.

    A point on an edge with a NaN end is NaN on both sides, but the bits of
    a NaN are not portable: x86 propagates the input NaN's payload
    (0x7fc00000 for numpy's nan) while CUDA arithmetic returns the canonical
    0x7fffffff.  NaN positions must match; every other coordinate must match
    bit for bit.
    """
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    assert a.shape == b.shape
    na, nb = np.isnan(a), np.isnan(b)
    np.testing.assert_array_equal(na, nb)
    np.testing.assert_array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))


def assert_same_surface(got, ref, exact_points=True):
    """Counts and conn exact; points bit-identical (or within 1e-5 rel)."""
    assert got["total_points"] == ref["total_points"]
    assert got["total_tris"] == ref["total_tris"]
    np.testing.assert_array_equal(got["conn"], ref["conn"])
    if exact_points:
        assert_points_identical(got["points"], ref["points"])
    else:
        a, b = got["points"].astype(np.float64), ref["points"].astype(np.float64)
        np.testing.assert_array_less(np.abs(a - b), np.maximum(1e-5 * np.abs(b), 1e-5) + 1e-30)
