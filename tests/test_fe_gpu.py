"""Flying edges on the GPU against the reference's own outputs.

Every golden fixture was produced by the reference (tack.cpu).  The GPU
result must be identical: totals, per-row offsets (scan), connectivity, and
point coordinates bit for bit (the kernels use the reference's f32
operation order without contraction; the 1e-5 relative tolerance allowed
for vertex positions is not needed).
"""

import numpy as np
import pytest

from conftest import GOLDEN, golden_fe_cases, load_fe_case
from fe_helpers import (assert_points_identical, assert_same_surface, capi_fe,
                        reference_offsets_from_rows)

pytestmark = pytest.mark.gpu


def _upload(tack, arr, dtype):
    f = tack.field(dtype, (arr.size,))
    f.from_numpy(arr)
    return f


@pytest.mark.parametrize("name", golden_fe_cases())
def test_api_matches_reference(tack, name):
    """tack_b200.flying_edges_multiblock == the reference's output."""
    c = load_fe_case(name)
    grid = tack.UniformGrid(*c["grid_tuple"])
    blk = {"scalar": _upload(tack, c["values"], tack.f32), "grid": grid}
    if c["mask"] is not None:
        blk["mask"] = _upload(tack, c["mask"], tack.i32)
    r = tack.flying_edges_multiblock([blk], c["isovalue"])
    if int(c["is_none"]):
        assert r is None
        return
    ref = {"total_points": int(c["totals"][0]), "total_tris": int(c["totals"][1]),
           "points": c["points"], "conn": c["conn"]}
    assert_same_surface(r, ref)
    assert r["block_point_counts"] == [ref["total_points"]]
    assert r["block_tri_counts"] == [ref["total_tris"]]
    assert_points_identical(r["points_field"].to_numpy().reshape(-1, 3), r["points"])
    np.testing.assert_array_equal(r["conn_field"].to_numpy().reshape(-1, 3), r["conn"])


@pytest.mark.parametrize("name", golden_fe_cases())
def test_capi_counts_and_offsets_match_reference(tack, name):
    """Through the raw C ABI: the scan offsets equal _count_block's."""
    c = load_fe_case(name)
    g = c["grid_tuple"]
    got = capi_fe(c["values"], g, [c["isovalue"]], c["mask"], want_rows=True)
    xo, yo, zo, to = reference_offsets_from_rows(got["rows"][0], got["counts"][0], g)
    np.testing.assert_array_equal(xo, c["xo"])
    np.testing.assert_array_equal(yo, c["yo"])
    np.testing.assert_array_equal(zo, c["zo"])
    np.testing.assert_array_equal(to, c["tri_offsets"])
    assert int(got["counts"][0, :3].sum()) == int(c["count_totals"][0])
    assert int(got["counts"][0, 3]) == int(c["count_totals"][1])
    if not int(c["is_none"]):
        ref = {"total_points": int(c["totals"][0]), "total_tris": int(c["totals"][1]),
               "points": c["points"], "conn": c["conn"]}
        assert_same_surface(got, ref)


def test_multiblock_matches_reference(tack):
    z = np.load(f"{GOLDEN}/fe_multiblock_sphere24.npz")
    blocks = []
    for b in (0, 1):
        g = z[f"grid{b}"]
        grid = tack.UniformGrid(int(g[0]), int(g[1]), int(g[2]), *g[3:])
        blocks.append({"scalar": _upload(tack, z[f"values{b}"], tack.f32), "grid": grid})
    r = tack.flying_edges_multiblock(blocks, 0.0)
    np.testing.assert_array_equal(r["conn"], z["conn"])
    assert_points_identical(r["points"], z["points"])
    assert r["block_point_counts"] == list(z["block_point_counts"])
    assert r["block_tri_counts"] == list(z["block_tri_counts"])


def test_isovalue_list_matches_per_isovalue_reference(tack, oracle):
    """A list of isovalues == the oracle's per-isovalue calls, concatenated."""
    c = load_fe_case("gyroid48")
    g = c["grid_tuple"]
    isos = [-0.5, -0.1, 0.0, 0.3, 0.7, 1.2, -1.0, 0.05, 0.5]  # 9: two groups
    f = _upload(tack, c["values"], tack.f32)
    r = tack.flying_edges(f, tack.UniformGrid(*g), isos)
    ref = oracle.flying_edges_isovalues(c["values"], oracle.Grid(*g), isos)
    assert_same_surface(r, ref)
    assert r["isovalue_point_counts"] == ref["isovalue_point_counts"]
    assert r["isovalue_tri_counts"] == ref["isovalue_tri_counts"]


def test_capi_multi_isovalue_one_read(tack, oracle):
    """tkmc_fe_count with 8 isovalues classifies all of them in one launch."""
    c = load_fe_case("blobs72")
    g = c["grid_tuple"]
    isos = [0.05, 0.1, 0.2, 0.3, 0.5, 0.7, 0.9, 1.1]
    got = capi_fe(c["values"], g, isos, want_rows=True)
    ref = oracle.flying_edges_isovalues(c["values"], oracle.Grid(*g), isos)
    assert_same_surface(got, ref)
    for q, iso in enumerate(isos):
        info = oracle.count_block(c["values"], oracle.Grid(*g), iso)
        xo, yo, zo, to = reference_offsets_from_rows(got["rows"][q], got["counts"][q], g)
        np.testing.assert_array_equal(xo, info["xo"])
        np.testing.assert_array_equal(yo, info["yo"])
        np.testing.assert_array_equal(zo, info["zo"])
        np.testing.assert_array_equal(to, info["tri_offsets"])


def test_fe_run_capacity_protocol(tack):
    """tkmc_fe_run: too-small buffers -> TKMC_ERR_CAPACITY with counts."""
    import ctypes

    import torch

    from fe_helpers import f32arr, stream
    from tack_b200 import _lib
    c = load_fe_case("c1_sphere64")
    nx, ny, nz = c["grid_tuple"][:3]
    lib = _lib.load()
    v = torch.from_numpy(c["values"]).cuda()
    nb = lib.tkmc_fe_workspace_bytes(nx, ny, nz, 1)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    counts = np.zeros(4, np.int64)
    pts = torch.empty(3 * 100, dtype=torch.float32, device="cuda")
    conn = torch.empty(3 * 100, dtype=torch.int32, device="cuda")
    rc = lib.tkmc_fe_run(v.data_ptr(), nx, ny, nz, f32arr(c["grid_tuple"][3:]), f32arr([0.0]), 1,
                         None, ws.data_ptr(), nb, pts.data_ptr(), 100, conn.data_ptr(), 100,
                         counts.ctypes.data, stream())
    assert rc == _lib.TKMC_ERR_CAPACITY
    assert int(counts[:3].sum()) == 7584 and int(counts[3]) == 15164
    P, T = int(counts[:3].sum()), int(counts[3])
    pts = torch.empty(3 * P, dtype=torch.float32, device="cuda")
    conn = torch.empty(3 * T, dtype=torch.int32, device="cuda")
    rc = lib.tkmc_fe_run(v.data_ptr(), nx, ny, nz, f32arr(c["grid_tuple"][3:]), f32arr([0.0]), 1,
                         None, ws.data_ptr(), nb, pts.data_ptr(), P, conn.data_ptr(), T,
                         counts.ctypes.data, stream())
    assert rc == 0
    np.testing.assert_array_equal(conn.cpu().numpy().reshape(-1, 3), c["conn"])
    assert_points_identical(pts.cpu().numpy().reshape(-1, 3), c["points"])
    del ctypes


def test_unaligned_volume_pointer(tack, oracle):
    """A volume that does not start on a 16-byte boundary (scalar loads)."""
    import torch
    c = load_fe_case("noise_19x13x11")
    g = c["grid_tuple"]
    buf = torch.empty(c["values"].size + 1, dtype=torch.float32, device="cuda")
    buf[1:] = torch.from_numpy(c["values"]).cuda()
    got = capi_fe(buf[1:], g, [c["isovalue"]])
    ref = {"total_points": int(c["totals"][0]), "total_tris": int(c["totals"][1]),
           "points": c["points"], "conn": c["conn"]}
    assert_same_surface(got, ref)


def test_reference_cuda_field_duck_typing(tack):
    """A field exposing only ._buffer.device_ptr and .shape (as tack.cuda's
    fields do) is accepted without a copy."""
    c = load_fe_case("sphere24_in")
    f = _upload(tack, c["values"], tack.f32)

    class Buf:
        device_ptr = f._buffer.device_ptr

    class RefField:
        _buffer = Buf()
        shape = f.shape

    r = tack.flying_edges(RefField(), tack.UniformGrid(*c["grid_tuple"]), 0.0)
    np.testing.assert_array_equal(r["conn"], c["conn"])


def test_empty_and_uniform_volumes(tack):
    g = tack.UniformGrid(7, 5, 3, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
    n = 8 * 6 * 4
    for val in (-1.0, 1.0, 0.0):
        f = _upload(tack, np.full(n, val, np.float32), tack.f32)
        assert tack.flying_edges(f, g, 0.0) is None
    f = _upload(tack, np.full(n, np.nan, np.float32), tack.f32)
    assert tack.flying_edges(f, g, 0.0) is None
    assert tack.flying_edges_multiblock([], 0.0) is None


def test_degenerate_grids_match_oracle(tack, oracle):
    """Grids with one or zero cells along an axis."""
    rng = np.random.default_rng(5)
    for shape in ((0, 4, 4), (4, 0, 4), (4, 4, 0), (1, 1, 1), (0, 0, 3), (33, 1, 0), (1, 40, 2)):
        nx, ny, nz = shape
        v = rng.standard_normal((nx + 1) * (ny + 1) * (nz + 1)).astype(np.float32)
        g = (nx, ny, nz, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
        got = tack.flying_edges(_upload(tack, v, tack.f32), tack.UniformGrid(*g), 0.0)
        ref = oracle.flying_edges(v, oracle.Grid(*g), 0.0)
        if ref is None:
            assert got is None
        else:
            assert_same_surface(got, ref)


@pytest.mark.parametrize("shape", [(1099, 3, 4), (2047, 4, 3), (1500, 5, 2), (4999, 2, 2),
                                   (9000, 2, 1), (1023, 2, 2), (1024, 3, 2)])
def test_long_rows_match_oracle(tack, oracle, shape):
    """Rows longer than 1024 nodes: several threads per row in the count
    pass, multi-word activity masks, and (beyond 8192 nodes) the row-wise
    emit kernel."""
    nx, ny, nz = shape
    rng = np.random.default_rng(nx)
    n = (nx + 1) * (ny + 1) * (nz + 1)
    # Smooth along x with sparse crossings plus a few dense stretches.
    i = np.arange(n) % (nx + 1)
    v = (np.sin(i * 0.013 + rng.random()) + 0.3 * rng.standard_normal(n)).astype(np.float32)
    g = (nx, ny, nz, 0.25, -1.0, 3.0, 0.5, 1.5, 0.75)
    for iso in (0.0, 0.9):
        got = capi_fe(v, g, [iso], want_rows=True)
        ref = oracle.flying_edges(v, oracle.Grid(*g), iso)
        info = oracle.count_block(v, oracle.Grid(*g), iso)
        xo, yo, zo, to = reference_offsets_from_rows(got["rows"][0], got["counts"][0], g)
        np.testing.assert_array_equal(xo, info["xo"])
        np.testing.assert_array_equal(yo, info["yo"])
        np.testing.assert_array_equal(zo, info["zo"])
        np.testing.assert_array_equal(to, info["tri_offsets"])
        if ref is None:
            assert got["total_points"] == 0 or got["total_tris"] == 0
        else:
            assert_same_surface(got, ref)


@pytest.mark.parametrize("shape,density", [((255, 127, 30), "noise"), ((127, 63, 40), "smooth"),
                                           ((2047, 6, 5), "smooth")])
def test_word_aligned_rows_unit_list(tack, oracle, shape, density):
    """Rows of a multiple of 32 nodes take the unit-list path: white noise
    (nearly every word active, rows with more active words than a warp's
    batch), smooth fields and long rows."""
    nx, ny, nz = shape
    assert (nx + 1) % 32 == 0
    rng = np.random.default_rng(nx + ny)
    n = (nx + 1) * (ny + 1) * (nz + 1)
    if density == "noise":
        v = rng.standard_normal(n).astype(np.float32)
    else:
        z, y, x = np.meshgrid(np.arange(nz + 1), np.arange(ny + 1), np.arange(nx + 1),
                              indexing="ij")
        v = (np.sin(x * 0.05) + np.cos(y * 0.11) * np.sin(z * 0.07)
             + 0.05 * rng.standard_normal(x.shape)).astype(np.float32).reshape(-1)
    g = (nx, ny, nz, -3.0, 0.5, 1.0, 0.1, 0.2, 0.3)
    for iso in (0.0, 0.4):
        got = capi_fe(v, g, [iso], want_rows=True)
        info = oracle.count_block(v, oracle.Grid(*g), iso)
        xo, yo, zo, to = reference_offsets_from_rows(got["rows"][0], got["counts"][0], g)
        np.testing.assert_array_equal(xo, info["xo"])
        np.testing.assert_array_equal(to, info["tri_offsets"])
        ref = oracle.flying_edges(v, oracle.Grid(*g), iso)
        assert_same_surface(got, ref)



@pytest.mark.parametrize("shape", [(2, 2, 2), (30, 20, 9), (159, 160, 161), (255, 255, 255),
                                   (1023, 3, 2)])
def test_volume_sizes_match_oracle(tack, oracle, shape):
    """Volumes of one to many 1024-node chunks per warp of the threshold
    pass, with ragged tails shorter than 16 bytes."""
    nx, ny, nz = shape
    n = (nx + 1) * (ny + 1) * (nz + 1)
    rng = np.random.default_rng(n % 1000)
    i = np.arange(n, dtype=np.int64)
    v = (np.sin(i % (nx + 1) * 0.07) + np.cos(i // ((nx + 1) * (ny + 1)) * 0.05)
         + 0.3 * rng.standard_normal(n)).astype(np.float32)
    g = (nx, ny, nz, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
    ref = oracle.flying_edges(v, oracle.Grid(*g), 0.4)
    got = capi_fe(v, g, [0.4])
    if ref is None:
        assert got["total_points"] == 0 or got["total_tris"] == 0
    else:
        assert_same_surface(got, ref)


def test_many_blocks_match_oracle(tack, oracle):
    """Many blocks of different shapes (word-aligned rows and not), some
    masked, some empty: counts of all blocks are read with one
    synchronisation, then every block emits; the concatenation equals the
    oracle's flying_edges_multiblock."""
    rng = np.random.default_rng(11)
    blocks_gpu, blocks_ref = [], []
    for b in range(40):
        nx, ny, nz = (31 if b % 3 else 20), int(rng.integers(2, 12)), int(rng.integers(1, 9))
        n = (nx + 1) * (ny + 1) * (nz + 1)
        v = (rng.standard_normal(n) + (5.0 if b % 7 == 0 else 0.0)).astype(np.float32)  # some empty
        g = (nx, ny, nz, float(b), 0.0, 0.0, 0.5, 0.5, 0.5)
        mask = None
        if b % 4 == 1:
            mask = (rng.random(nx * ny * nz) < 0.3).astype(np.int32)
        blk = {"scalar": _upload(tack, v, tack.f32), "grid": tack.UniformGrid(*g)}
        ref = {"values": v, "grid": oracle.Grid(*g)}
        if mask is not None:
            blk["mask"] = _upload(tack, mask, tack.i32)
            ref["mask"] = mask
        blocks_gpu.append(blk)
        blocks_ref.append(ref)
    r = tack.flying_edges_multiblock(blocks_gpu, 0.2)
    ref = oracle.flying_edges_multiblock(blocks_ref, 0.2)
    np.testing.assert_array_equal(r["conn"], ref["conn"])
    assert_points_identical(r["points"], ref["points"])
    assert r["block_point_counts"] == list(ref["block_point_counts"])
    assert r["block_tri_counts"] == list(ref["block_tri_counts"])


@pytest.mark.parametrize("cells,nblocks", [((31, 31, 31), 27), ((32, 32, 32), 27), ((7, 5, 3), 200)])
def test_block_batches_match_oracle(tack, oracle, cells, nblocks):
    """Blocks of one shape go through the batched count and emit (rows of a
    multiple of 32 nodes and not, tiny blocks of one partial chunk), with
    masks on some blocks and several isovalues; equal to the oracle's
    flying_edges_multiblock per isovalue, concatenated."""
    nx, ny, nz = cells
    rng = np.random.default_rng(nx * 7 + nblocks)
    n = (nx + 1) * (ny + 1) * (nz + 1)
    blocks_gpu, blocks_ref = [], []
    for b in range(nblocks):
        i = np.arange(n)
        v = (np.sin(i * 0.013 + b) + 0.4 * rng.standard_normal(n)).astype(np.float32)
        g = (nx, ny, nz, float(b % 3) * nx, float(b // 3 % 3) * ny, float(b // 9) * nz,
             0.5, 0.75, 1.0)
        blk = {"scalar": _upload(tack, v, tack.f32), "grid": tack.UniformGrid(*g)}
        ref = {"values": v, "grid": oracle.Grid(*g)}
        if b % 5 == 2:
            m = (rng.random(nx * ny * nz) < 0.4).astype(np.int32)
            blk["mask"] = _upload(tack, m, tack.i32)
            ref["mask"] = m
        blocks_gpu.append(blk)
        blocks_ref.append(ref)
    isos = [0.1, -0.5]
    r = tack.flying_edges_multiblock(blocks_gpu, isos)
    pts, conns, p0 = [], [], 0
    for iso in isos:
        ref = oracle.flying_edges_multiblock(blocks_ref, iso)
        pts.append(ref["points"])
        conns.append(ref["conn"] + p0)
        p0 += ref["points"].shape[0]
    np.testing.assert_array_equal(r["conn"], np.concatenate(conns))
    assert_points_identical(r["points"], np.concatenate(pts))


def test_amr_blanking_style_masks_match_oracle(tack, oracle):
    """Masks as amr_blanking.build_masks (amr_blanking.py:26) writes them:
    per-cell flags DUPLICATECELL = 1 (ghost layers), REFINEDCELL = 8 (covered
    by a finer level) and both (9).  Any nonzero flag removes the cell's
    triangles (flying_edges.py:441-477); points stay.  Word-aligned and
    ragged row lengths, one block through flying_edges_multiblock."""
    from tack_b200 import workloads
    for shape in ((64, 48, 40), (70, 33, 29)):
        nx, ny, nz = shape[0] - 1, shape[1] - 1, shape[2] - 1
        v = workloads.generate("gyroid", shape).cpu().numpy()
        mask = np.zeros((nz, ny, nx), np.int32)
        mask[:2] |= 1                 # ghost layers at both z ends and one y side
        mask[-2:] |= 1
        mask[:, :2] |= 1
        mask[10:20, 8:24, 5:40] |= 8  # a refined box, overlapping a ghost layer
        mask = mask.reshape(-1)
        g = (nx, ny, nz, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
        blk = {"scalar": _upload(tack, v, tack.f32), "grid": tack.UniformGrid(*g),
               "mask": _upload(tack, mask, tack.i32)}
        got = tack.flying_edges_multiblock([blk], 0.0)
        ref = oracle.flying_edges(v, oracle.Grid(*g), 0.0, mask)
        np.testing.assert_array_equal(got["conn"], ref["conn"])
        assert_points_identical(got["points"], ref["points"])
        plain = oracle.flying_edges(v, oracle.Grid(*g), 0.0)
        assert ref["total_tris"] < plain["total_tris"]
        assert ref["total_points"] == plain["total_points"]
