"""CPU parity oracle for the flying-edges isosurface path.

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
as the checker, and by ``bench.py`` for its CPU-baseline leg and reference
arm.  The product path (``tack_b200``) never imports it.

The kernels are the C restatement in ``fe_oracle.c`` (built to
``oracle/liboracle_fe.so``); this module restates the reference's host
orchestration around them:

* ``count_block``  -- flying_edges.py:663-715 (_count_block): count kernels,
  then numpy sums and cumsums into row offsets (kept int64 here).
* ``emit_block``   -- flying_edges.py:718-746 (_emit_block).
* ``flying_edges`` / ``flying_edges_multiblock`` -- flying_edges.py:749-832,
  same result dict, ``None`` when there are no points or no triangles.
* ``classify_cells``  -- 26_marching_cubes.py:435-450 (per-cell case, count).
* ``scan`` -- scan.py:81-123; ``reduce`` -- field.py:116-134.

The marching-cubes tables are the reference's own, dumped into
``tests/golden/mc_tables.npz`` by ``tests/golden/make_golden.py``.

Parity status: pinned.  ``tests/test_oracle_golden.py`` checks this oracle
against outputs of the reference itself (``tests/golden/*.npz``).
"""

import ctypes
import os
import subprocess

import numpy as np

ORACLE_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(ORACLE_DIR)
LIB_PATH = os.path.join(ORACLE_DIR, "liboracle_fe.so")
SRC_PATH = os.path.join(ORACLE_DIR, "fe_oracle.c")
TABLES_PATH = os.path.join(REPO_DIR, "tests", "golden", "mc_tables.npz")

CFLAGS = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-pthread",
          "-std=c11"]


def build(force=False, verbose=False):
    """Compile fe_oracle.c into liboracle_fe.so (gcc, no external deps)."""
    if (not force and os.path.exists(LIB_PATH)
            and os.path.getmtime(LIB_PATH) >= os.path.getmtime(SRC_PATH)):
        return LIB_PATH
    cmd = ["gcc", *CFLAGS, SRC_PATH, "-o", LIB_PATH + ".tmp", "-lm"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


class _Grid(ctypes.Structure):
    _fields_ = [("nx", ctypes.c_int64), ("ny", ctypes.c_int64), ("nz", ctypes.c_int64),
                ("x0", ctypes.c_float), ("y0", ctypes.c_float), ("z0", ctypes.c_float),
                ("dx", ctypes.c_float), ("dy", ctypes.c_float), ("dz", ctypes.c_float)]


_lib = None
_tables = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        I64, F, I = ctypes.c_int64, ctypes.c_float, ctypes.c_int
        G = ctypes.POINTER(_Grid)
        L.orc_fe_count_edges_xyz.argtypes = [P, G, F, P, P, P, I]
        L.orc_fe_count_rows.argtypes = [P, G, P, P, F, P, I]
        L.orc_fe_emit_points_xyz.argtypes = [P, P, P, P, P, G, F, I]
        L.orc_fe_emit_tris.argtypes = [P, P, P, P, P, P, P, G, P, F, I]
        L.orc_mc_classify_cells.argtypes = [P, G, P, F, P, P, I]
        L.orc_scan_i32.argtypes = [P, P, I64, I]
        L.orc_scan_i32.restype = I64
        L.orc_reduce_f32.argtypes = [P, I64, P]
        L.orc_mc_soup.argtypes = [P, G, P, P, F, P, P, P, P, I]
        L.orc_mc_soup.restype = None
        L.orc_compute_normals.argtypes = [P, P, I64, I64, P]
        L.orc_compute_normals.restype = None
        L.orc_num_threads.argtypes = [I]
        L.orc_num_threads.restype = I
        for name in ("orc_fe_count_edges_xyz", "orc_fe_count_rows", "orc_fe_emit_points_xyz",
                     "orc_fe_emit_tris", "orc_mc_classify_cells", "orc_reduce_f32"):
            getattr(L, name).restype = None
        _lib = L
    return _lib


def tables():
    """The reference's (tri_table[4096], num_tris[256], edge_corners[24])."""
    global _tables
    if _tables is None:
        z = np.load(TABLES_PATH)
        _tables = (np.ascontiguousarray(z["tri_table"], np.int32),
                   np.ascontiguousarray(z["num_tris"], np.int32),
                   np.ascontiguousarray(z["edge_corners"], np.int32))
    return _tables


def num_threads(n=0):
    return lib().orc_num_threads(int(n))


class Grid:
    """UniformGrid(nx, ny, nz, x0, y0, z0, dx, dy, dz) (flying_edges.py:313-341)."""

    def __init__(self, nx, ny, nz, x0=0.0, y0=0.0, z0=0.0, dx=1.0, dy=1.0, dz=1.0):
        self.nx, self.ny, self.nz = int(nx), int(ny), int(nz)
        self.x0, self.y0, self.z0 = x0, y0, z0
        self.dx, self.dy, self.dz = dx, dy, dz

    @classmethod
    def of(cls, g):
        return cls(g.nx, g.ny, g.nz, g.x0, g.y0, g.z0, g.dx, g.dy, g.dz)

    def c(self):
        f = lambda x: float(np.float32(x))  # kernel scalars are f32
        return _Grid(self.nx, self.ny, self.nz, f(self.x0), f(self.y0), f(self.z0),
                     f(self.dx), f(self.dy), f(self.dz))


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _f32(values, grid):
    v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    n = (grid.nx + 1) * (grid.ny + 1) * (grid.nz + 1)
    if v.size != n:
        raise ValueError(f"field has {v.size} values, grid needs {n}")
    return v


def count_block(values, grid, isovalue, mask=None, nthreads=0):
    """_count_block: row counts, totals and intra-block row offsets (int64)."""
    g = Grid.of(grid)
    v = _f32(values, g)
    iso = np.float32(isovalue)
    nnr = (g.ny + 1) * (g.nz + 1)
    ncr = g.ny * g.nz
    xc = np.zeros(nnr, np.int32)
    yc = np.zeros(nnr, np.int32)
    zc = np.zeros(nnr, np.int32)
    tri = np.zeros(ncr, np.int32)
    gc = g.c()
    m = None if mask is None else np.ascontiguousarray(mask, np.int32).reshape(-1)
    L = lib()
    L.orc_fe_count_edges_xyz(_ptr(v), ctypes.byref(gc), iso, _ptr(xc), _ptr(yc), _ptr(zc),
                             nthreads)
    L.orc_fe_count_rows(_ptr(v), ctypes.byref(gc), _ptr(tables()[1]), _ptr(m), iso, _ptr(tri),
                        nthreads)
    tx, ty, tz = int(xc.sum(dtype=np.int64)), int(yc.sum(dtype=np.int64)), int(zc.sum(dtype=np.int64))
    tt = int(tri.sum(dtype=np.int64))
    xo = np.zeros(nnr, np.int64)
    yo = np.zeros(nnr, np.int64)
    zo = np.zeros(nnr, np.int64)
    to = np.zeros(ncr, np.int64)
    xo[1:] = np.cumsum(xc[:-1], dtype=np.int64)
    yo[1:] = np.cumsum(yc[:-1], dtype=np.int64)
    yo += tx
    zo[1:] = np.cumsum(zc[:-1], dtype=np.int64)
    zo += tx + ty
    if ncr:
        to[1:] = np.cumsum(tri[:-1], dtype=np.int64)
    return {"n_node_rows": nnr, "n_cell_rows": ncr, "row_xc": xc, "row_yc": yc, "row_zc": zc,
            "row_tri": tri, "total_x": tx, "total_y": ty, "total_z": tz,
            "total_points": tx + ty + tz, "total_tris": tt,
            "xo": xo, "yo": yo, "zo": zo, "tri_offsets": to}


def emit_block(values, grid, isovalue, info, pt_offset, tri_offset, points, conn, mask=None,
               nthreads=0):
    """_emit_block: write points (flat f32) and conn (flat i32) at the offsets."""
    g = Grid.of(grid)
    v = _f32(values, g)
    iso = np.float32(isovalue)
    xo = np.ascontiguousarray(info["xo"] + pt_offset, np.int64)
    yo = np.ascontiguousarray(info["yo"] + pt_offset, np.int64)
    zo = np.ascontiguousarray(info["zo"] + pt_offset, np.int64)
    to = np.ascontiguousarray(info["tri_offsets"] + tri_offset, np.int64)
    gc = g.c()
    m = None if mask is None else np.ascontiguousarray(mask, np.int32).reshape(-1)
    L = lib()
    L.orc_fe_emit_points_xyz(_ptr(v), _ptr(xo), _ptr(yo), _ptr(zo), _ptr(points),
                             ctypes.byref(gc), iso, nthreads)
    if info["n_cell_rows"]:
        L.orc_fe_emit_tris(_ptr(v), _ptr(to), _ptr(xo), _ptr(yo), _ptr(zo), _ptr(conn), _ptr(m),
                           ctypes.byref(gc), _ptr(tables()[0]), iso, nthreads)


def flying_edges_multiblock(blocks, isovalue, nthreads=0):
    """flying_edges_multiblock (flying_edges.py:766-832) on host arrays.

    blocks: list of dicts with 'values' (f32 array), 'grid' and optional 'mask'.
    """
    if len(blocks) == 0:
        return None
    infos = [count_block(b["values"], b["grid"], isovalue, b.get("mask"), nthreads)
             for b in blocks]
    pt_off = np.zeros(len(blocks), np.int64)
    tri_off = np.zeros(len(blocks), np.int64)
    for b in range(1, len(blocks)):
        pt_off[b] = pt_off[b - 1] + infos[b - 1]["total_points"]
        tri_off[b] = tri_off[b - 1] + infos[b - 1]["total_tris"]
    total_points = int(pt_off[-1] + infos[-1]["total_points"])
    total_tris = int(tri_off[-1] + infos[-1]["total_tris"])
    if total_points == 0 or total_tris == 0:
        return None
    points = np.zeros(total_points * 3, np.float32)
    conn = np.zeros(total_tris * 3, np.int32)
    for b, blk in enumerate(blocks):
        if infos[b]["total_points"] == 0:
            continue
        emit_block(blk["values"], blk["grid"], isovalue, infos[b], int(pt_off[b]),
                   int(tri_off[b]), points, conn, blk.get("mask"), nthreads)
    return {"points": points.reshape(-1, 3), "conn": conn.reshape(-1, 3),
            "total_points": total_points, "total_tris": total_tris,
            "block_point_counts": [int(i["total_points"]) for i in infos],
            "block_tri_counts": [int(i["total_tris"]) for i in infos],
            "infos": infos}


def flying_edges(values, grid, isovalue, mask=None, nthreads=0):
    """flying_edges (flying_edges.py:749-763) on a host array."""
    blk = {"values": values, "grid": grid}
    if mask is not None:
        blk["mask"] = mask
    return flying_edges_multiblock([blk], isovalue, nthreads)


def flying_edges_isovalues(values, grid, isovalues, mask=None, nthreads=0):
    """One flying_edges call per isovalue, concatenated: each isovalue's conn
    is offset by the points of the isovalues before it (the multi-block
    concatenation rule of flying_edges.py:797-832 applied across isovalues)."""
    pts, conns, pc, tc = [], [], [], []
    base = 0
    for iso in isovalues:
        r = flying_edges(values, grid, iso, mask, nthreads)
        if r is None:
            pc.append(0)
            tc.append(0)
            continue
        pts.append(r["points"])
        conns.append(r["conn"] + base)
        pc.append(r["total_points"])
        tc.append(r["total_tris"])
        base += r["total_points"]
    if sum(pc) == 0 or sum(tc) == 0:
        return None
    return {"points": np.concatenate(pts), "conn": np.concatenate(conns),
            "total_points": sum(pc), "total_tris": sum(tc),
            "isovalue_point_counts": pc, "isovalue_tri_counts": tc}


def classify_cells(values, grid, isovalue, nthreads=0):
    """Per-cell case index (uint8) and triangle count (int32)."""
    g = Grid.of(grid)
    v = _f32(values, g)
    n = g.nx * g.ny * g.nz
    cases = np.zeros(n, np.uint8)
    ntri = np.zeros(n, np.int32)
    gc = g.c()
    lib().orc_mc_classify_cells(_ptr(v), ctypes.byref(gc), _ptr(tables()[1]),
                                np.float32(isovalue), _ptr(cases), _ptr(ntri), nthreads)
    return cases, ntri


def scan(values, inclusive=False):
    """Prefix sum of int32 values (int32 output with wrap); returns (out, total)."""
    a = np.ascontiguousarray(values, np.int32).reshape(-1)
    out = np.zeros_like(a)
    total = lib().orc_scan_i32(_ptr(a), _ptr(out), a.size, 1 if inclusive else 0)
    return out, int(total)


def reduce(values):
    """(min, max, sum, nan_count) of f32 values; min/max ignore NaN."""
    a = np.ascontiguousarray(values, np.float32).reshape(-1)
    out = np.zeros(4, np.float64)
    lib().orc_reduce_f32(_ptr(a), a.size, _ptr(out))
    return float(out[0]), float(out[1]), float(out[2]), int(out[3])


def compute_normals(points, conn):
    """Vertex normals of a triangle mesh (compute_normals.py:16-90): f32
    (n_pts, 3).  points (n_pts, 3) f32, conn (n_tris, 3) int32."""
    p = np.ascontiguousarray(points, np.float32).reshape(-1)
    c = np.ascontiguousarray(conn, np.int32).reshape(-1)
    n_pts, n_tris = p.size // 3, c.size // 3
    out = np.zeros(3 * n_pts, np.float32)
    lib().orc_compute_normals(_ptr(p), _ptr(c), n_pts, n_tris, _ptr(out))
    return out.reshape(-1, 3)


def mc_soup(values, grid, isovalue, nthreads=0):
    """classify_cells + exclusive_scan + emit_triangles of
    examples/26_marching_cubes.py:435-503: the unmerged triangle soup as
    SoA f32 arrays (x, y, z) of 3*T vertices, and T."""
    g = Grid.of(grid)
    v = _f32(values, g)
    cases, ntri = classify_cells(v, g, isovalue, nthreads)
    off = np.zeros(ntri.size, np.int64)
    if ntri.size:
        off[1:] = np.cumsum(ntri[:-1], dtype=np.int64)
    total = int(ntri.sum(dtype=np.int64))
    out = [np.zeros(max(3 * total, 1), np.float32) for _ in range(3)]
    tri, _, edges = tables()
    gc = g.c()
    lib().orc_mc_soup(_ptr(v), ctypes.byref(gc), _ptr(tri), _ptr(edges), np.float32(isovalue),
                      _ptr(off), _ptr(out[0]), _ptr(out[1]), _ptr(out[2]), nthreads)
    return out[0][:3 * total], out[1][:3 * total], out[2][:3 * total], total
