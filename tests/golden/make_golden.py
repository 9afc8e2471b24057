"""Generate the golden fixtures in tests/golden/ by running the reference.

Runs berkgeveci/tack's own code on its CPU backend (tack.cpu, llvmlite JIT)
and records inputs and outputs as .npz files.  The reference is imported
from a source checkout of berkgeveci/tack given by ``--reference`` or, when
that is omitted, by the environment variable TACK_REFERENCE (read-only;
nothing is written there).  The fixtures are committed; the tests never need
the reference itself.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <checkout>

What is recorded (all through the reference's public or module-level API):
  mc_tables.npz     _TRI_TABLE, _NUM_TRIS, _EDGE_CORNERS (flying_edges.py:33-306)
  fe_<case>.npz     input volume, grid, isovalue, mask; the reference's
                    flying_edges result (points, conn, totals) and its
                    _count_block row counts and offsets (flying_edges.py:663-715)
  mc_classify.npz   per-cell triangle counts from examples/26_marching_cubes.py
                    classify_cells, their exclusive_scan offsets, and the
                    unmerged triangle soup of its emit_triangles
  scan.npz          tack.algorithms.exclusive_scan / inclusive_scan outputs
  reduce.npz        Field.sum/min/max outputs on tack.cpu
  normals.npz       tack.algorithms.compute_normals on small meshes, a random
                    mesh and a flying-edges sphere (compute_normals.py:16-90)
"""

import argparse
import hashlib
import importlib
import os
import runpy
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(root):
    sys.path[:0] = [os.path.join(root, "packages", "tack-core", "src"),
                    os.path.join(root, "packages", "tack-vis", "src")]
    import tack  # noqa: E402
    tack.init(tack.cpu)
    return tack


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---------------------------------------------------------------- volumes

def node_coords(nx, ny, nz, x0, y0, z0, dx, dy, dz):
    i, j, k = np.arange(nx + 1), np.arange(ny + 1), np.arange(nz + 1)
    kk, jj, ii = np.meshgrid(k, j, i, indexing="ij")
    return (x0 + ii * dx).ravel(), (y0 + jj * dy).ravel(), (z0 + kk * dz).ravel()


def sphere_sdf64():
    """64^3 nodes: distance to (31.5,31.5,31.5) minus 20, unit spacing."""
    i = np.arange(64, dtype=np.float64)
    kk, jj, ii = np.meshgrid(i, i, i, indexing="ij")
    r = np.sqrt((ii - 31.5) ** 2 + (jj - 31.5) ** 2 + (kk - 31.5) ** 2)
    return (r - 20.0).astype(np.float32).ravel()


def cube_grid(n, lo=-1.5, hi=1.5):
    h = (hi - lo) / n
    return (n, n, n, lo, lo, lo, h, h, h)


def sphere_values(g, radius=1.0, inside_positive=True):
    x, y, z = node_coords(*g)
    r2 = x * x + y * y + z * z
    v = radius ** 2 - r2 if inside_positive else r2 - radius ** 2
    return v.astype(np.float32)


def noise_values(g, seed, iso, nan_frac=0.0, tie_frac=0.0):
    """Uniform noise with some nodes exactly at the isovalue and some NaN."""
    rng = np.random.default_rng(seed)
    n = (g[0] + 1) * (g[1] + 1) * (g[2] + 1)
    v = (rng.random(n) * 2.0 - 1.0).astype(np.float32)
    if tie_frac:
        v[rng.random(n) < tie_frac] = np.float32(iso)
    if nan_frac:
        v[rng.random(n) < nan_frac] = np.nan
    return v


def blobs_values(g, seed, nblobs=6):
    rng = np.random.default_rng(seed)
    x, y, z = node_coords(*g)
    v = np.zeros(x.shape, np.float64)
    for _ in range(nblobs):
        c = rng.uniform(0, [g[0], g[1], g[2]])
        s = rng.uniform(3, 9)
        w = rng.uniform(0.5, 1.5)
        v += w * np.exp(-((x - c[0]) ** 2 + (y - c[1]) ** 2 + (z - c[2]) ** 2) / (2 * s * s))
    return v.astype(np.float32)


def gyroid_values(n, seed):
    """Gyroid with x,y,z = 2*pi*4*index/n plus N(0, 0.01) noise (n nodes/axis)."""
    t = 2 * np.pi * 4 * np.arange(n) / n
    zz, yy, xx = np.meshgrid(t, t, t, indexing="ij")
    v = np.sin(xx) * np.cos(yy) + np.sin(yy) * np.cos(zz) + np.sin(zz) * np.cos(xx)
    v = v + np.random.default_rng(seed).normal(0.0, 0.01, v.shape)
    return v.astype(np.float32).ravel()


# ---------------------------------------------------------------- cases

def fe_cases():
    """(name, values, grid tuple, isovalue, mask or None)."""
    cases = []
    cases.append(("c1_sphere64", sphere_sdf64(), (63, 63, 63, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0),
                  0.0, None))
    g = (4, 4, 4, 0.0, 0.0, 0.0, 0.25, 0.25, 0.25)
    cases.append(("plane4", node_coords(*g)[2].astype(np.float32), g, 0.375, None))
    g = cube_grid(24)
    cases.append(("sphere24_in", sphere_values(g), g, 0.0, None))
    cases.append(("sphere24_out", sphere_values(g, inside_positive=False), g, 0.0, None))
    for t in (0.6, 0.8):
        cases.append((f"sphere24_iso{int(t * 10)}", sphere_values(g), g, 1.0 - t * t, None))
    for n in (2, 3, 5):
        g = cube_grid(n)
        cases.append((f"tiny{n}", sphere_values(g), g, 0.0, None))
    g = (20, 24, 16, 2.0, -5.0, 10.0, 0.1, 0.25, 0.125)
    x, y, z = node_coords(*g)
    v = (0.36 - ((x - 3.0) ** 2 + (y + 2.0) ** 2 + (z - 11.0) ** 2)).astype(np.float32)
    cases.append(("aniso", v, g, 0.0, None))
    g = cube_grid(16)
    m = np.zeros(16 ** 3, np.int32)
    m[: 16 ** 3 // 2] = 1
    cases.append(("masked16", sphere_values(g), g, 0.0, m))
    m2 = (np.random.default_rng(7).random(16 ** 3) < 0.3).astype(np.int32)
    cases.append(("masked16_rand", sphere_values(g), g, 0.0, m2))
    # Row lengths around 32-bit word boundaries, non-cubic, ties and NaNs.
    for (nx, ny, nz), seed in (((32, 7, 5), 11), ((63, 4, 3), 12), ((64, 5, 4), 13),
                               ((31, 3, 2), 14), ((95, 6, 3), 15), ((19, 13, 11), 16),
                               ((1, 9, 7), 17), ((40, 1, 1), 18)):
        g = (nx, ny, nz, 0.5, -0.25, 1.0, 0.75, 1.25, 0.5)
        cases.append((f"noise_{nx}x{ny}x{nz}", noise_values(g, seed, 0.1, 0.02, 0.05), g, 0.1,
                      None))
    g = (47, 47, 47, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
    cases.append(("gyroid48", gyroid_values(48, 3), g, 0.0, None))
    g = (71, 59, 66, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
    cases.append(("blobs72", blobs_values(g, 5), g, 0.5, None))
    g = cube_grid(12)
    cases.append(("all_below", np.full(13 ** 3, -1.0, np.float32), g, 0.0, None))
    cases.append(("iso_at_max", sphere_values(g), g, float(np.float32(1.0)), None))
    return cases


def run_fe(tack, name, values, g, iso, mask, out_dir):
    fe_mod = importlib.import_module("tack.algorithms.flying_edges")
    grid = fe_mod.UniformGrid(*g)
    f = tack.field(dtype=tack.f32, shape=(values.size,))
    f.from_numpy(values)
    blk = {"scalar": f, "grid": grid}
    m = None
    if mask is not None:
        m = tack.field(dtype=tack.i32, shape=(mask.size,))
        m.from_numpy(mask)
        blk["mask"] = m
    res = fe_mod.flying_edges_multiblock([blk], iso)
    if m is None:
        m = tack.field(dtype=tack.i32, shape=(g[0] * g[1] * g[2],))
        m.fill(0)
    info = fe_mod._count_block(f, grid, iso, m)
    rec = {
        "values": values, "grid": np.array(g, np.float64), "isovalue": np.float64(iso),
        "mask": mask if mask is not None else np.zeros(0, np.int32),
        "has_mask": np.int32(mask is not None),
        "is_none": np.int32(res is None),
        "xo": info["xo_np"], "yo": info["yo_np"], "zo": info["zo_np"],
        "tri_offsets": info["tri_offsets_np"],
        "count_totals": np.array([info["total_points"], info["total_tris"]], np.int64),
    }
    if res is not None:
        rec.update(points=res["points"], conn=res["conn"],
                   totals=np.array([res["total_points"], res["total_tris"]], np.int64))
    np.savez_compressed(os.path.join(out_dir, f"fe_{name}.npz"), **rec)
    return res


def run_multiblock(tack, out_dir):
    """tests/test_flying_edges.py:_split_sphere_blocks -- two z-stacked blocks."""
    fe_mod = importlib.import_module("tack.algorithms.flying_edges")
    n, half = 24, 12
    h = 3.0 / n
    grids = [(n, n, half, -1.5, -1.5, -1.5, h, h, h),
             (n, n, half, -1.5, -1.5, -1.5 + half * h, h, h, h)]
    vals = [sphere_values(g) for g in grids]
    blocks = []
    for g, v in zip(grids, vals):
        f = tack.field(dtype=tack.f32, shape=(v.size,))
        f.from_numpy(v)
        blocks.append({"scalar": f, "grid": fe_mod.UniformGrid(*g)})
    res = fe_mod.flying_edges_multiblock(blocks, 0.0)
    np.savez_compressed(os.path.join(out_dir, "fe_multiblock_sphere24.npz"),
                        values0=vals[0], values1=vals[1],
                        grid0=np.array(grids[0], np.float64), grid1=np.array(grids[1], np.float64),
                        points=res["points"], conn=res["conn"],
                        totals=np.array([res["total_points"], res["total_tris"]], np.int64),
                        block_point_counts=np.array(res["block_point_counts"], np.int64),
                        block_tri_counts=np.array(res["block_tri_counts"], np.int64))


def run_mc_classify(tack, root, out_dir):
    """Per-cell counts from example 26's classify_cells + exclusive_scan."""
    from tack import algorithms
    saved = sys.argv
    sys.argv = ["26_marching_cubes.py", "--size", "4", "--warmup", "0", "--trials", "1"]
    try:
        ex = runpy.run_path(os.path.join(root, "packages", "tack-vis", "examples",
                                         "26_marching_cubes.py"),
                            run_name="tack_example_26")
    finally:
        sys.argv = saved
    rec = {}
    for name, values, g, iso in (("c1", sphere_sdf64(), (63, 63, 63, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0), 0.0),
                                 ("noise", noise_values((19, 13, 11), 16, 0.1, 0.02, 0.05),
                                  (19, 13, 11, 0.5, -0.25, 1.0, 0.75, 1.25, 0.5), 0.1),
                                 ("aligned", noise_values((63, 9, 5), 23, -0.2, 0.01, 0.02),
                                  (63, 9, 5, -3.0, 2.0, 0.125, 0.3, 0.7, 1.1), -0.2)):
        grid = ex["UniformGrid3D"](*g)
        tables = ex["MCTables"]()
        n_cells = g[0] * g[1] * g[2]
        f = tack.field(dtype=tack.f32, shape=(values.size,))
        f.from_numpy(values)
        num_tri = tack.field(dtype=tack.i32, shape=(n_cells,))
        ex["classify_cells"](f, num_tri, grid, tables, n_cells, iso)
        offsets = tack.field(dtype=tack.i32, shape=(n_cells,))
        total = algorithms.exclusive_scan(num_tri, offsets, n_cells)
        rec[f"{name}_values"] = values
        rec[f"{name}_grid"] = np.array(g, np.float64)
        rec[f"{name}_iso"] = np.float64(iso)
        rec[f"{name}_num_tri"] = num_tri.to_numpy()
        rec[f"{name}_offsets"] = offsets.to_numpy()
        rec[f"{name}_total"] = np.int64(total)
        # The unmerged triangle soup of emit_triangles (SoA x, y, z).
        outs = [tack.field(dtype=tack.f32, shape=(max(3 * total, 1),)) for _ in range(3)]
        ex["emit_triangles"](f, offsets, grid, tables, *outs, n_cells, iso)
        for axis, o in zip("xyz", outs):
            rec[f"{name}_soup_{axis}"] = o.to_numpy()[:3 * total]
    np.savez_compressed(os.path.join(out_dir, "mc_classify.npz"), **rec)


def run_scan(tack, out_dir):
    from tack import algorithms
    vecs = {
        "basic": np.array([3, 1, 4, 1, 5, 9, 2, 6], np.int32),
        "ones100": np.ones(100, np.int32),
        "zeros16": np.zeros(16, np.int32),
        "pow2_16": np.arange(1, 17, dtype=np.int32),
        "n37": np.arange(1, 38, dtype=np.int32),
        "ones64": np.ones(64, np.int32),
        "rand5000": np.random.default_rng(21).integers(0, 6, 5000).astype(np.int32),
    }
    rec = {}
    for k, v in vecs.items():
        n = v.size
        inp = tack.field(dtype=tack.i32, shape=(n,))
        inp.from_numpy(v)
        out = tack.field(dtype=tack.i32, shape=(n,))
        tot = algorithms.exclusive_scan(inp, out, n)
        rec[f"{k}_in"] = v
        rec[f"{k}_excl"] = out.to_numpy()
        rec[f"{k}_excl_total"] = np.int64(tot)
        out2 = tack.field(dtype=tack.i32, shape=(n,))
        tot2 = algorithms.inclusive_scan(inp, out2, n)
        rec[f"{k}_incl"] = out2.to_numpy()
        rec[f"{k}_incl_total"] = np.int64(tot2)
    np.savez_compressed(os.path.join(out_dir, "scan.npz"), **rec)


def run_reduce(tack, out_dir):
    rng = np.random.default_rng(31)
    vecs = {"arange8": np.arange(8, dtype=np.float32),
            "rand10001": rng.standard_normal(10001).astype(np.float32),
            "sphere64": sphere_sdf64()}
    rec = {}
    for k, v in vecs.items():
        f = tack.field(dtype=tack.f32, shape=(v.size,))
        f.from_numpy(v)
        rec[f"{k}_in"] = v
        rec[f"{k}_out"] = np.array([f.min(), f.max(), f.sum()], np.float64)
    np.savez_compressed(os.path.join(out_dir, "reduce.npz"), **rec)


def normals_cases():
    """Meshes for compute_normals: the kinds the reference's tests use
    (one triangle either winding, a flat quad, two faces folded 90 degrees,
    a big and a tiny face sharing a vertex, a vertex no face touches, a
    zero-area face), a flying-edges sphere, and a random shared-vertex mesh."""
    cases = {
        "tri_ccw": (np.array([[0, 0, 0], [1, 0, 0], [0, 1, 0]]), np.array([[0, 1, 2]])),
        "tri_cw": (np.array([[0, 0, 0], [1, 0, 0], [0, 1, 0]]), np.array([[0, 2, 1]])),
        "quad": (np.array([[0, 0, 0], [2, 0, 0], [2, 3, 0], [0, 3, 0]]),
                 np.array([[0, 1, 2], [0, 2, 3]])),
        "fold": (np.array([[0, 0, 0], [1, 0, 0], [1, 1, 0], [0, 1, 0], [0, 0, 1], [0, 1, 1]]),
                 np.array([[0, 1, 2], [0, 2, 3], [0, 5, 3], [0, 4, 5]])),
        "big_small": (np.array([[0, 0, 0], [8, 0, 0], [0, 8, 0], [0, 0, 0.02], [0, 0.02, 0]]),
                      np.array([[0, 1, 2], [0, 3, 4]])),
        "unreferenced": (np.array([[0, 0, 0], [1, 0, 0], [0, 1, 0], [4, 4, 4]]),
                         np.array([[0, 1, 2]])),
        "degenerate": (np.array([[0, 0, 0], [1, 0, 0], [3, 0, 0]]), np.array([[0, 1, 2]])),
    }
    rng = np.random.default_rng(41)
    pts = rng.standard_normal((2000, 3))
    tris = np.stack([rng.permutation(2000)[:3] for _ in range(6000)])
    cases["random"] = (pts, tris)
    return {k: (np.asarray(p, np.float32), np.asarray(c, np.int32)) for k, (p, c) in cases.items()}


def run_normals(tack, out_dir):
    """compute_normals on each mesh (tack.algorithms.compute_normals), and on
    the flying-edges surface of fe_sphere24_in's volume."""
    cn = importlib.import_module("tack.algorithms.compute_normals")
    fe_mod = importlib.import_module("tack.algorithms.flying_edges")
    meshes = normals_cases()
    g = cube_grid(24)
    v = sphere_values(g)
    f = tack.field(dtype=tack.f32, shape=(v.size,))
    f.from_numpy(v)
    r = fe_mod.flying_edges(f, fe_mod.UniformGrid(*g), 0.0)
    meshes["fe_sphere24"] = (r["points"].astype(np.float32), r["conn"].astype(np.int32))
    rec = {}
    for k, (p, c) in meshes.items():
        pf = tack.field(dtype=tack.f32, shape=(p.size,))
        pf.from_numpy(p.reshape(-1))
        cf = tack.field(dtype=tack.i32, shape=(c.size,))
        cf.from_numpy(c.reshape(-1))
        out = cn.compute_normals(pf, cf, p.shape[0], c.shape[0])
        rec[f"{k}_points"] = p
        rec[f"{k}_conn"] = c
        rec[f"{k}_normals"] = out.to_numpy().reshape(-1, 3)
    np.savez_compressed(os.path.join(out_dir, "normals.npz"), **rec)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TACK_REFERENCE"),
                    help="source checkout of berkgeveci/tack (default: $TACK_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    if not a.reference:
        ap.error("give the reference checkout with --reference or TACK_REFERENCE")
    tack = load_reference(a.reference)
    fe_mod = importlib.import_module("tack.algorithms.flying_edges")
    np.savez_compressed(os.path.join(a.out, "mc_tables.npz"), tri_table=fe_mod._TRI_TABLE,
                        num_tris=fe_mod._NUM_TRIS, edge_corners=fe_mod._EDGE_CORNERS)
    manifest = []
    for name, values, g, iso, mask in fe_cases():
        res = run_fe(tack, name, values, g, iso, mask, a.out)
        tot = None if res is None else (res["total_points"], res["total_tris"])
        manifest.append(f"fe_{name}: input sha256 {sha(values)[:16]} -> {tot}")
    run_multiblock(tack, a.out)
    run_mc_classify(tack, a.reference, a.out)
    run_scan(tack, a.out)
    run_reduce(tack, a.out)
    run_normals(tack, a.out)
    with open(os.path.join(a.out, "MANIFEST.txt"), "w") as fh:
        fh.write("Generated by tests/golden/make_golden.py from the reference on tack.cpu.\n")
        fh.write("\n".join(manifest) + "\n")
    print("\n".join(manifest))


if __name__ == "__main__":
    main()
