"""Pin the CPU oracle to the reference's own outputs.

Every fixture in tests/golden/ was produced by running berkgeveci/tack on
tack.cpu (tests/golden/make_golden.py).  The oracle must reproduce each one
exactly: counts, offsets, connectivity, and point coordinates bit for bit.
"""

import numpy as np
import pytest

from conftest import GOLDEN, golden_fe_cases, load_fe_case


@pytest.mark.parametrize("name", golden_fe_cases())
def test_oracle_matches_reference(oracle, name):
    c = load_fe_case(name)
    g = oracle.Grid(*c["grid_tuple"])
    r = oracle.flying_edges(c["values"], g, c["isovalue"], c["mask"])
    if int(c["is_none"]):
        assert r is None
        return
    assert r is not None
    assert (r["total_points"], r["total_tris"]) == tuple(c["totals"])
    np.testing.assert_array_equal(r["conn"], c["conn"])
    np.testing.assert_array_equal(r["points"].view(np.uint32), c["points"].view(np.uint32))
    info = r["infos"][0]
    np.testing.assert_array_equal(info["xo"], c["xo"])
    np.testing.assert_array_equal(info["yo"], c["yo"])
    np.testing.assert_array_equal(info["zo"], c["zo"])
    np.testing.assert_array_equal(info["tri_offsets"], c["tri_offsets"])


def test_oracle_multiblock_matches_reference(oracle):
    z = np.load(f"{GOLDEN}/fe_multiblock_sphere24.npz")
    blocks = [{"values": z["values0"], "grid": oracle.Grid(*z["grid0"][:3].astype(int), *z["grid0"][3:])},
              {"values": z["values1"], "grid": oracle.Grid(*z["grid1"][:3].astype(int), *z["grid1"][3:])}]
    r = oracle.flying_edges_multiblock(blocks, 0.0)
    np.testing.assert_array_equal(r["conn"], z["conn"])
    np.testing.assert_array_equal(r["points"].view(np.uint32), z["points"].view(np.uint32))
    assert r["block_point_counts"] == list(z["block_point_counts"])
    assert r["block_tri_counts"] == list(z["block_tri_counts"])


@pytest.mark.parametrize("name", ["c1", "noise", "aligned"])
def test_oracle_per_cell_counts_and_offsets(oracle, name):
    """classify_cells + exclusive_scan of examples/26_marching_cubes.py, and
    its emit_triangles soup bit for bit."""
    z = np.load(f"{GOLDEN}/mc_classify.npz")
    g = z[f"{name}_grid"]
    grid = oracle.Grid(int(g[0]), int(g[1]), int(g[2]), *g[3:])
    cases, ntri = oracle.classify_cells(z[f"{name}_values"], grid, float(z[f"{name}_iso"]))
    np.testing.assert_array_equal(ntri, z[f"{name}_num_tri"])
    off, total = oracle.scan(ntri)
    np.testing.assert_array_equal(off, z[f"{name}_offsets"])
    assert total == int(z[f"{name}_total"])
    # case index -> count through the reference's table
    np.testing.assert_array_equal(oracle.tables()[1][cases], ntri)
    x, y, zc, t = oracle.mc_soup(z[f"{name}_values"], grid, float(z[f"{name}_iso"]))
    assert t == int(z[f"{name}_total"])
    for got, ax in ((x, "x"), (y, "y"), (zc, "z")):
        np.testing.assert_array_equal(got.view(np.uint32), z[f"{name}_soup_{ax}"].view(np.uint32))


def test_oracle_scan_known_answers(oracle):
    z = np.load(f"{GOLDEN}/scan.npz")
    keys = sorted({k.rsplit("_", 1)[0] for k in z.files if k.endswith("_in")})
    assert "basic" in keys
    for k in keys:
        out, tot = oracle.scan(z[f"{k}_in"])
        np.testing.assert_array_equal(out, z[f"{k}_excl"])
        assert tot == int(z[f"{k}_excl_total"])
        out, tot = oracle.scan(z[f"{k}_in"], inclusive=True)
        np.testing.assert_array_equal(out, z[f"{k}_incl"])
        assert tot == int(z[f"{k}_incl_total"])
    # test_algorithms.py:9-22 known answer
    out, tot = oracle.scan(np.array([3, 1, 4, 1, 5, 9, 2, 6], np.int32))
    assert list(out) == [0, 3, 4, 8, 9, 14, 23, 25] and tot == 31


def test_oracle_reductions(oracle):
    z = np.load(f"{GOLDEN}/reduce.npz")
    for k in ("arange8", "rand10001", "sphere64"):
        mn, mx, sm, nan = oracle.reduce(z[f"{k}_in"])
        ref = z[f"{k}_out"]
        assert mn == ref[0] and mx == ref[1] and nan == 0
        assert sm == pytest.approx(ref[2], rel=1e-5, abs=1e-3)
    mn, mx, sm, _ = oracle.reduce(np.arange(8, dtype=np.float32))
    assert (mn, mx, sm) == (0.0, 7.0, 28.0)  # test_backend_contract.py:102-118


def test_oracle_thread_count_does_not_change_output(oracle):
    c = load_fe_case("gyroid48")
    g = oracle.Grid(*c["grid_tuple"])
    a = oracle.flying_edges(c["values"], g, c["isovalue"], nthreads=1)
    b = oracle.flying_edges(c["values"], g, c["isovalue"], nthreads=7)
    np.testing.assert_array_equal(a["conn"], b["conn"])
    np.testing.assert_array_equal(a["points"], b["points"])


def test_oracle_normals_match_reference(oracle):
    """compute_normals.py:16-90 restated: the reference's normals on every
    fixture mesh (small meshes of its tests' kinds, a random mesh, a
    flying-edges sphere), bit for bit."""
    z = np.load(f"{GOLDEN}/normals.npz")
    names = sorted({k.rsplit("_", 1)[0] for k in z.files})
    assert len(names) >= 9
    for n in names:
        got = oracle.compute_normals(z[f"{n}_points"], z[f"{n}_conn"])
        np.testing.assert_array_equal(got.view(np.uint32), z[f"{n}_normals"].view(np.uint32), n)
