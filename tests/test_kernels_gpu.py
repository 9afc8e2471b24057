"""Scan, field reductions and per-cell classification on the GPU.

Known answers come from the reference's own tests and fixtures
(tests/golden/scan.npz, reduce.npz, mc_classify.npz); larger cases are
checked against the oracle.
"""

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _field(tack, arr, dtype):
    f = tack.field(dtype, (arr.size,))
    f.from_numpy(arr)
    return f


def test_scan_known_answers(tack):
    z = np.load(f"{GOLDEN}/scan.npz")
    keys = sorted({k.rsplit("_", 1)[0] for k in z.files if k.endswith("_in")})
    for k in keys:
        a = z[f"{k}_in"]
        inp, out = _field(tack, a, tack.i32), tack.field(tack.i32, (a.size,))
        tot = tack.algorithms.exclusive_scan(inp, out, a.size)
        np.testing.assert_array_equal(out.to_numpy(), z[f"{k}_excl"])
        assert tot == int(z[f"{k}_excl_total"])
        tot = tack.algorithms.inclusive_scan(inp, out, a.size)
        np.testing.assert_array_equal(out.to_numpy(), z[f"{k}_incl"])
        assert tot == int(z[f"{k}_incl_total"])
        np.testing.assert_array_equal(inp.to_numpy(), a)  # input preserved


@pytest.mark.parametrize("n", [1, 31, 4095, 4096, 4097, 1 << 20, 3_000_017])
def test_scan_sizes_match_oracle(tack, oracle, n):
    a = np.random.default_rng(n).integers(-50, 1000, n).astype(np.int32)
    inp, out = _field(tack, a, tack.i32), tack.field(tack.i32, (n,))
    tot = tack.algorithms.exclusive_scan(inp, out, n)
    ref, rtot = oracle.scan(a)
    np.testing.assert_array_equal(out.to_numpy(), ref)
    assert tot == rtot


def test_scan_wraps_like_int32_and_aliases(tack, oracle):
    a = np.full(50_000, 2_000_000_000 // 7, np.int32)
    f = _field(tack, a, tack.i32)
    tot = tack.algorithms.inclusive_scan(f, f, a.size)  # in place
    ref, rtot = oracle.scan(a, inclusive=True)
    np.testing.assert_array_equal(f.to_numpy(), ref)
    assert tot == rtot == int(a.astype(np.int64).sum())


def test_reductions_contract(tack):
    """test_backend_contract.py:102-118: 0..7 -> 28 / 0 / 7."""
    f = _field(tack, np.arange(8, dtype=np.float32), tack.f32)
    assert f.sum() == pytest.approx(28.0)
    assert f.min() == 0.0 and f.max() == 7.0
    assert f.mean() == pytest.approx(3.5)


def test_reductions_match_reference_fixtures(tack):
    z = np.load(f"{GOLDEN}/reduce.npz")
    for k in ("arange8", "rand10001", "sphere64"):
        f = _field(tack, z[f"{k}_in"], tack.f32)
        ref = z[f"{k}_out"]
        assert f.min() == ref[0] and f.max() == ref[1]
        assert f.sum() == pytest.approx(ref[2], rel=1e-5, abs=1e-3)


@pytest.mark.parametrize("offset", [0, 1, 2, 3])
def test_reductions_large_unaligned_with_nan(tack, oracle, offset):
    n = 5_000_003
    a = np.random.default_rng(9).standard_normal(n + offset).astype(np.float32)
    a[offset + 12345] = np.nan
    a[offset + 777] = 9.5
    a[-1] = -11.25
    t = torch.from_numpy(a).cuda()[offset:]
    mn, mx, sm, nan = tack.reduce_f32(t)
    rmn, rmx, rsm, rnan = oracle.reduce(a[offset:])
    assert (mn, mx, nan) == (rmn, rmx, rnan) == (-11.25, 9.5, 1)
    assert np.isnan(sm) and np.isnan(rsm)


def test_reduction_sum_accuracy(tack):
    a = np.random.default_rng(3).random(10_000_000).astype(np.float32)
    f = _field(tack, a, tack.f32)
    assert f.sum() == pytest.approx(float(a.astype(np.float64).sum()), rel=1e-12)


def test_classify_cells_matches_reference(tack):
    """Per-cell counts of examples/26_marching_cubes.py classify_cells and
    their exclusive_scan offsets."""
    z = np.load(f"{GOLDEN}/mc_classify.npz")
    for name in ("c1", "noise"):
        g = z[f"{name}_grid"]
        grid = tack.UniformGrid(int(g[0]), int(g[1]), int(g[2]), *g[3:])
        f = _field(tack, z[f"{name}_values"], tack.f32)
        cases, ntri = tack.algorithms.classify_cells(f, grid, float(z[f"{name}_iso"]))
        np.testing.assert_array_equal(ntri.to_numpy(), z[f"{name}_num_tri"])
        off = tack.field(tack.i32, ntri.shape)
        tot = tack.algorithms.exclusive_scan(ntri, off, ntri.size)
        np.testing.assert_array_equal(off.to_numpy(), z[f"{name}_offsets"])
        assert tot == int(z[f"{name}_total"])


def test_classify_cases_match_oracle(tack, oracle):
    from conftest import load_fe_case
    c = load_fe_case("noise_95x6x3")
    g = c["grid_tuple"]
    f = _field(tack, c["values"], tack.f32)
    cases, ntri = tack.algorithms.classify_cells(f, tack.UniformGrid(*g), c["isovalue"])
    rc, rn = oracle.classify_cells(c["values"], oracle.Grid(*g), c["isovalue"])
    np.testing.assert_array_equal(cases.to_numpy(), rc)
    np.testing.assert_array_equal(ntri.to_numpy(), rn)


def _nan_aware_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    assert a.shape == b.shape
    na, nb = np.isnan(a), np.isnan(b)
    np.testing.assert_array_equal(na, nb)
    np.testing.assert_array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))


def test_soup_matches_reference(tack):
    """marching_cubes_soup == example 26's emit_triangles, vertex for vertex
    (rows of a multiple of 32 nodes and not, NaNs and ties at the isovalue)."""
    z = np.load(f"{GOLDEN}/mc_classify.npz")
    for name in ("c1", "noise", "aligned"):
        g = z[f"{name}_grid"]
        grid = tack.UniformGrid(int(g[0]), int(g[1]), int(g[2]), *g[3:])
        f = _field(tack, z[f"{name}_values"], tack.f32)
        r = tack.algorithms.marching_cubes_soup(f, grid, float(z[f"{name}_iso"]))
        assert r["total_tris"] == int(z[f"{name}_total"])
        for ax in "xyz":
            _nan_aware_equal(r[ax], z[f"{name}_soup_{ax}"])


@pytest.mark.parametrize("shape", [(95, 60, 41), (100, 37, 30), (2047, 4, 3)])
def test_soup_matches_oracle(tack, oracle, shape):
    """Larger grids, several isovalues and a mask, against the oracle's
    restatement of example 26."""
    nx, ny, nz = shape
    rng = np.random.default_rng(nx)
    zz, yy, xx = np.meshgrid(np.arange(nz + 1), np.arange(ny + 1), np.arange(nx + 1), indexing="ij")
    v = (np.sin(xx * 0.11) + np.cos(yy * 0.23) * np.sin(zz * 0.19)
         + 0.1 * rng.standard_normal(xx.shape)).astype(np.float32).reshape(-1)
    g = (nx, ny, nz, 0.25, -1.0, 2.0, 0.5, 0.3, 0.7)
    isos = [0.0, 0.6]
    r = tack.algorithms.marching_cubes_soup(_field(tack, v, tack.f32), tack.UniformGrid(*g), isos)
    for q, iso in enumerate(isos):
        x, y, zc, total = oracle.mc_soup(v, oracle.Grid(*g), iso)
        assert r["isovalue_tri_counts"][q] == total
        lo = 3 * sum(r["isovalue_tri_counts"][:q])
        for ax, ref in zip("xyz", (x, y, zc)):
            _nan_aware_equal(r[ax][lo:lo + 3 * total], ref)
    mask = (rng.random(nx * ny * nz) < 0.5).astype(np.int32)
    rm = tack.algorithms.marching_cubes_soup(_field(tack, v, tack.f32), tack.UniformGrid(*g), 0.0,
                                             mask=_field(tack, mask, tack.i32))
    x, y, zc, total = oracle.mc_soup(v, oracle.Grid(*g), 0.0)
    _, ntri = oracle.classify_cells(v, oracle.Grid(*g), 0.0)
    keep = np.repeat(mask == 0, 3 * ntri)  # the soup without the masked cells' triangles
    assert rm["total_tris"] == int(ntri[mask == 0].sum())
    _nan_aware_equal(rm["x"], x[keep])


def test_copy_counts_to_device_pinned_and_pageable_memory(tack):
    """tkmc_fe_copy_counts writes the same totals whether the destination is
    this GPU's memory or page-locked host memory (a kernel store) or pageable
    host memory (a copy), and they equal tkmc_fe_read_counts'."""
    import ctypes
    from tack_b200 import _lib, workloads
    from fe_helpers import f32arr, stream
    lib = _lib.load()
    shape = (128, 96, 80)
    nx, ny, nz = shape[0] - 1, shape[1] - 1, shape[2] - 1
    vol = workloads.generate("blobs", shape)
    isos = [0.5, 0.9, 0.2]
    nb = lib.tkmc_fe_workspace_bytes(nx, ny, nz, len(isos))
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    want = np.zeros(4 * len(isos), np.int64)
    _lib.check(lib.tkmc_fe_count(vol.data_ptr(), nx, ny, nz, 0, f32arr(isos), len(isos), None,
                                 ws.data_ptr(), nb, want.ctypes.data, stream()), "count")
    assert want.sum() > 0
    dev = torch.full((4 * len(isos),), -1, dtype=torch.int64, device="cuda")
    pinned = torch.full((4 * len(isos),), -1, dtype=torch.int64, pin_memory=True)
    pageable = np.full(4 * len(isos), -1, np.int64)
    for ptr in (dev.data_ptr(), pinned.data_ptr(), pageable.ctypes.data):
        _lib.check(lib.tkmc_fe_copy_counts(nx, ny, nz, len(isos), ws.data_ptr(), nb, ptr,
                                           stream()), "copy_counts")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dev.cpu().numpy(), want)
    np.testing.assert_array_equal(pinned.numpy(), want)
    np.testing.assert_array_equal(pageable, want)
    del ctypes
