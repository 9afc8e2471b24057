"""Flying edges isosurface (merged-point marching cubes) on sm_100a.

Drop-in for packages/tack-vis/src/tack/algorithms/flying_edges.py: the same
``flying_edges(scalar, grid, isovalue)`` and
``flying_edges_multiblock(blocks, isovalue)`` entry points, the same
``UniformGrid`` descriptor and ``MCTables``, and the same result dict
(``points``, ``conn``, ``points_field``, ``conn_field``, ``total_points``,
``total_tris``, ``block_point_counts``, ``block_tri_counts``; ``None`` when
the surface is empty).  Points, connectivity, counts and offsets are
bit-identical to the reference's.

Differences, all extensions:

* ``isovalue`` may be a sequence: each isovalue's points and triangles
  follow the previous one's (conn offset by the points before it), and the
  dict adds ``isovalue_point_counts`` / ``isovalue_tri_counts``.  Up to 8
  isovalues share one read of the volume.
* Without a ``mask`` no zero mask is allocated (the reference allocates and
  fills a 4 B/cell mask per call, flying_edges.py:783-788) and the block
  dicts are not modified.
* ``copy_to_host=False`` skips the device->host copies; ``points`` and
  ``conn`` are then ``None`` and the fields hold the result.

Each call: one ``tkmc_fe_count`` per block and group of <= 8 isovalues (one
volume read + a single-pass scan + a 32-byte-per-isovalue host read of the
totals), exact-size output allocation, one ``tkmc_fe_emit``.
"""

import ctypes
from collections.abc import Sequence

import numpy as np
import torch

from .. import _lib
from ..field import Field, CUDABuffer, device_tensor, f32, field, i32
from ..runtime import current_device, current_stream, workspace

__all__ = ["UniformGrid", "MCTables", "flying_edges", "flying_edges_multiblock",
           "_TRI_TABLE", "_NUM_TRIS", "_EDGE_CORNERS"]


def _load_tables():
    tri = np.zeros(4096, np.int32)
    num = np.zeros(256, np.int32)
    edges = np.zeros(24, np.int32)
    _lib.check(_lib.load().tkmc_mc_tables(tri.ctypes.data, num.ctypes.data, edges.ctypes.data),
               "tkmc_mc_tables")
    return tri, num, edges


_TABLE_NAMES = ("_TRI_TABLE", "_NUM_TRIS", "_EDGE_CORNERS")
_tables = None


def __getattr__(name):
    """_TRI_TABLE, _NUM_TRIS, _EDGE_CORNERS: the case tables the kernels use,
    read back from the library on first access."""
    global _tables
    if name in _TABLE_NAMES:
        if _tables is None:
            _tables = dict(zip(_TABLE_NAMES, _load_tables()))
        return _tables[name]
    raise AttributeError(name)


class UniformGrid:
    """Uniform grid descriptor: nx, ny, nz cells, origin and spacing.

    Same constructor and attributes as flying_edges.py:313-341.
    """

    def __init__(self, nx, ny, nz, x0, y0, z0, dx, dy, dz):
        self.nx = nx
        self.ny = ny
        self.nz = nz
        self.nx_p1 = nx + 1
        self.ny_p1 = ny + 1
        self.nxy_p1 = (nx + 1) * (ny + 1)
        self.x0 = x0
        self.y0 = y0
        self.z0 = z0
        self.dx = dx
        self.dy = dy
        self.dz = dz

    def get_x(self, i, j, k):
        return float(np.float32(self.x0) + np.float32(i) * np.float32(self.dx))

    def get_y(self, i, j, k):
        return float(np.float32(self.y0) + np.float32(j) * np.float32(self.dy))

    def get_z(self, i, j, k):
        return float(np.float32(self.z0) + np.float32(k) * np.float32(self.dz))

    @property
    def n_nodes(self):
        return (self.nx + 1) * (self.ny + 1) * (self.nz + 1)

    @property
    def n_cells(self):
        return self.nx * self.ny * self.nz



class MCTables:
    """Marching-cubes lookup tables as device fields (flying_edges.py:344-357).

    The kernels read their own copy from constant memory; these fields exist
    for callers that use the tables directly.
    """

    def __init__(self):
        tri, num, _ = _load_tables()
        self.tri_table = field(i32, (4096,))
        self.tri_table.from_numpy(tri)
        self.num_tris = field(i32, (256,))
        self.num_tris.from_numpy(num)


def _isovalue_list(isovalue):
    if isinstance(isovalue, (str, bytes)):
        raise TypeError("isovalue must be a number or a sequence of numbers")
    if isinstance(isovalue, (Sequence, np.ndarray, torch.Tensor)):
        vals = [float(v) for v in (isovalue.tolist() if hasattr(isovalue, "tolist") else isovalue)]
        if not vals:
            raise ValueError("empty list of isovalues")
        return vals, True
    return [float(isovalue)], False


def _geom6(g):
    """{x0, y0, z0, dx, dy, dz} of any grid with UniformGrid's attributes."""
    return (ctypes.c_float * 6)(g.x0, g.y0, g.z0, g.dx, g.dy, g.dz)


def _f32_array(vals):
    return (ctypes.c_float * len(vals))(*vals)


def _i64_array(vals):
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


class _Block:
    def __init__(self, blk, idx):
        self.idx = idx
        if "scalar" not in blk or "grid" not in blk:
            raise KeyError(f"block {idx} needs 'scalar' and 'grid'")
        self.grid = blk["grid"]
        g = self.grid
        if min(g.nx, g.ny, g.nz) < 0:
            raise ValueError(f"block {idx}: negative grid size")
        self.scalar = device_tensor(blk["scalar"], f32)
        n_nodes = (g.nx + 1) * (g.ny + 1) * (g.nz + 1)
        if self.scalar.numel() != n_nodes:
            raise ValueError(f"block {idx}: field has {self.scalar.numel()} values, grid needs "
                             f"{n_nodes}")
        m = blk.get("mask")
        self.mask = None if m is None else device_tensor(m, i32)
        if self.mask is not None and self.mask.numel() != g.nx * g.ny * g.nz:
            raise ValueError(f"block {idx}: mask has {self.mask.numel()} values, grid has "
                             f"{g.nx * g.ny * g.nz} cells")
        self.counts = []  # per isovalue group: (host int64 [niso*4], workspace)


class _Single:
    """One block counted and emitted on its own."""

    def __init__(self, block):
        self.block = block
        self.members = [block.idx]
        self.size = 1
        self.ws = {}

    def count(self, lib, grp, gi, counts_ptr, status_ptr, stream, dev, cached_ws):
        b, g = self.block, self.block.grid
        nbytes = lib.tkmc_fe_workspace_bytes(g.nx, g.ny, g.nz, len(grp))
        if nbytes == 0:
            raise ValueError(f"unsupported grid {g.nx} x {g.ny} x {g.nz}")
        ws = (workspace("fe", nbytes, dev) if cached_ws
              else torch.empty(nbytes, dtype=torch.uint8, device=dev))
        self.ws[gi] = ws
        mptr = b.mask.data_ptr() if b.mask is not None else None
        isoc = _f32_array(grp)
        _lib.check(lib.tkmc_fe_classify(b.scalar.data_ptr(), g.nx, g.ny, g.nz, isoc, len(grp),
                                        ws.data_ptr(), ws.numel(), stream), "tkmc_fe_classify")
        _lib.check(lib.tkmc_fe_scan(g.nx, g.ny, g.nz, 0, len(grp), mptr, ws.data_ptr(),
                                    ws.numel(), stream), "tkmc_fe_scan")
        _lib.check(lib.tkmc_fe_copy_counts(g.nx, g.ny, g.nz, len(grp), ws.data_ptr(), ws.numel(),
                                           counts_ptr, stream), "tkmc_fe_copy_counts")
        _lib.check(lib.tkmc_fe_copy_status(g.nx, g.ny, g.nz, len(grp), ws.data_ptr(), ws.numel(),
                                           status_ptr, stream), "tkmc_fe_copy_status")

    def emit(self, lib, grp, gi, bases, points_t, total_points, conn_t, total_tris, status_ptr,
             stream, dev):
        b, g, ws = self.block, self.block.grid, self.ws[gi]
        ida = _i64_array(bases[0, :, 0:3].reshape(-1))
        _lib.check(lib.tkmc_fe_emit(
            b.scalar.data_ptr(), g.nx, g.ny, g.nz, 0, 0, _geom6(g), _f32_array(grp), len(grp),
            b.mask.data_ptr() if b.mask is not None else None, ws.data_ptr(), ws.numel(), ida, ida,
            _i64_array(bases[0, :, 6]), points_t.data_ptr(), total_points, conn_t.data_ptr(),
            total_tris, stream), "tkmc_fe_emit")
        _lib.check(lib.tkmc_fe_copy_status(g.nx, g.ny, g.nz, len(grp), ws.data_ptr(), ws.numel(),
                                           status_ptr, stream), "tkmc_fe_copy_status")


class _Batch:
    """Blocks of one grid shape: one launch per phase for all of them."""

    def __init__(self, blocks, members, dev):
        self.members = list(members)
        self.size = len(members)
        bs = [blocks[i] for i in members]
        self.grid = bs[0].grid
        self.vols = torch.tensor([b.scalar.data_ptr() for b in bs], dtype=torch.int64).to(dev)
        has_mask = any(b.mask is not None for b in bs)
        self.masks = (torch.tensor([b.mask.data_ptr() if b.mask is not None else 0 for b in bs],
                                   dtype=torch.int64).to(dev) if has_mask else None)
        self.geoms = torch.tensor([[b.grid.x0, b.grid.y0, b.grid.z0, b.grid.dx, b.grid.dy,
                                    b.grid.dz] for b in bs], dtype=torch.float32).to(dev)
        self.ws = {}

    def count(self, lib, grp, gi, counts_ptr, status_ptr, stream, dev, cached_ws):
        g = self.grid
        stride = lib.tkmc_fe_batch_stride(g.nx, g.ny, g.nz, len(grp))
        if stride == 0:
            raise ValueError(f"unsupported grid {g.nx} x {g.ny} x {g.nz}")
        ws = torch.empty(stride * self.size, dtype=torch.uint8, device=dev)
        self.ws[gi] = ws
        _lib.check(lib.tkmc_fe_count_batch(
            self.vols.data_ptr(), self.size, g.nx, g.ny, g.nz, _f32_array(grp), len(grp),
            self.masks.data_ptr() if self.masks is not None else None, ws.data_ptr(), ws.numel(),
            counts_ptr, status_ptr, stream), "tkmc_fe_count_batch")

    def emit(self, lib, grp, gi, bases, points_t, total_points, conn_t, total_tris, status_ptr,
             stream, dev):
        g, ws = self.grid, self.ws[gi]
        bases_d = torch.from_numpy(np.ascontiguousarray(bases)).to(dev)
        _lib.check(lib.tkmc_fe_emit_batch(
            self.vols.data_ptr(), self.size, g.nx, g.ny, g.nz, self.geoms.data_ptr(),
            _f32_array(grp), len(grp), self.masks.data_ptr() if self.masks is not None else None,
            ws.data_ptr(), ws.numel(), bases_d.data_ptr(), points_t.data_ptr(), total_points,
            conn_t.data_ptr(), total_tris, status_ptr, stream), "tkmc_fe_emit_batch")
        self.bases_d = bases_d  # alive until the stream has used it


def _raise_status(status, phase):
    """Raise for the first device status word that records an error."""
    bad = np.nonzero(status)[0]
    if bad.size:
        code = int(status[bad[0]])
        what = ("device wait expired" if code == _lib.TKMC_ERR_DEVICE_TIMEOUT else
                "output capacity exceeded" if code == _lib.TKMC_ERR_CAPACITY else "error")
        raise _lib.TkmcError(code, f"flying edges {phase}: {what} (status {code})")


def flying_edges(scalar, grid, isovalue, *, copy_to_host=True):
    """Isosurface a single uniform grid block.

    Args:
        scalar: f32 field of node values, (nx+1)*(ny+1)*(nz+1) values with i
            fastest (a tack_b200 Field, a torch CUDA tensor, a reference tack
            field on its CUDA backend, or a host array: a numpy array or CPU
            tensor is copied to the device first, asynchronously when the
            tensor is pinned).
        grid: UniformGrid.
        isovalue: threshold, or a sequence of thresholds.

    Returns:
        dict with 'points' (numpy f32 (n,3)), 'conn' (numpy i32 (m,3)),
        'points_field', 'conn_field', 'total_points', 'total_tris', ...;
        None if empty.
    """
    return flying_edges_multiblock([{"scalar": scalar, "grid": grid}], isovalue,
                                   copy_to_host=copy_to_host)


def flying_edges_multiblock(blocks, isovalue, *, copy_to_host=True):
    """Isosurface a list of uniform grid blocks into one output.

    Args:
        blocks: list of dicts with 'scalar' and 'grid', optionally 'mask'
            (int32 per cell; nonzero cells emit no triangles).
        isovalue: threshold, or a sequence of thresholds.

    Returns:
        dict as flying_edges(); blocks (and isovalues) are concatenated in
        order, each block's conn offset by the points before it.  None if
        there are no points or no triangles.

    Blocks that share a grid shape are counted and emitted as one batch (one
    launch per phase for all of them); every block's totals are read with one
    synchronisation before the output is allocated.
    """
    if len(blocks) == 0:
        return None
    isos, is_list = _isovalue_list(isovalue)
    lib = _lib.load()
    dev = current_device()
    stream = current_stream(dev)
    bl = [_Block(b, i) for i, b in enumerate(blocks)]
    groups = [isos[i:i + _lib.MAX_ISO] for i in range(0, len(isos), _lib.MAX_ISO)]
    niso, nblk = len(isos), len(bl)

    # Parts: a batch of >= 2 blocks of one shape (at most 65535), or one block.
    by_shape = {}
    for bi, b in enumerate(bl):
        by_shape.setdefault((b.grid.nx, b.grid.ny, b.grid.nz), []).append(bi)
    parts = []
    for members in by_shape.values():
        for lo in range(0, len(members), 65535):
            chunk = members[lo:lo + 65535]
            parts.append(_Batch(bl, chunk, dev) if len(chunk) > 1 else _Single(bl[chunk[0]]))
    single_ws = len(parts) == 1 and len(groups) == 1 and isinstance(parts[0], _Single)

    # Pass 1: count every (part, isovalue group), totals and status words to
    # pinned host memory, then ONE synchronisation.
    counts_h = torch.zeros(nblk * niso * 4, dtype=torch.int64, pin_memory=True)
    status_h = torch.zeros(2 * nblk * niso, dtype=torch.int64, pin_memory=True)
    cnt = counts_h.numpy()
    slot = {}  # (part index, group index) -> row offset in counts_h / status_h (in int64s)
    row = 0
    for pi, part in enumerate(parts):
        for gi, grp in enumerate(groups):
            slot[(pi, gi)] = row
            part.count(lib, grp, gi, counts_h.data_ptr() + 8 * 4 * row,
                       status_h.data_ptr() + 8 * row, stream, dev, single_ws)
            row += part.size * len(grp)
    torch.cuda.current_stream(dev).synchronize()
    _raise_status(status_h.numpy()[:nblk * niso], "count")

    # Layout: isovalue-major, then block, then the X | Y | Z sections.
    pts = np.zeros((niso, nblk, 3), np.int64)
    tris = np.zeros((niso, nblk), np.int64)
    for pi, part in enumerate(parts):
        for gi, grp in enumerate(groups):
            c = cnt[4 * slot[(pi, gi)]:4 * (slot[(pi, gi)] + part.size * len(grp))]
            c = c.reshape(part.size, len(grp), 4)
            for k, bi in enumerate(part.members):
                for q in range(len(grp)):
                    qi = gi * _lib.MAX_ISO + q
                    pts[qi, bi] = c[k, q, :3]
                    tris[qi, bi] = c[k, q, 3]
    block_pts = pts.sum(axis=2)  # [iso, block]
    total_points = int(block_pts.sum())
    total_tris = int(tris.sum())
    if total_points == 0 or total_tris == 0:
        return None
    if total_points > 0x7FFFFFFF:
        raise OverflowError(f"{total_points} points do not fit int32 point ids")
    start_pt = np.concatenate([[0], np.cumsum(block_pts.reshape(-1))[:-1]]).reshape(niso, nblk)
    start_tri = np.concatenate([[0], np.cumsum(tris.reshape(-1))[:-1]]).reshape(niso, nblk)

    points_t = torch.empty(total_points * 3, dtype=torch.float32, device=dev)
    conn_t = torch.empty(total_tris * 3, dtype=torch.int32, device=dev)

    # Pass 2: emit every (part, isovalue group); status words after it.
    status_e = status_h.data_ptr() + 8 * nblk * niso
    row = 0
    for pi, part in enumerate(parts):
        for gi, grp in enumerate(groups):
            bases = np.zeros((part.size, len(grp), 7), np.int64)
            for k, bi in enumerate(part.members):
                for q in range(len(grp)):
                    qi = gi * _lib.MAX_ISO + q
                    p0 = start_pt[qi, bi]
                    X, Y = pts[qi, bi, 0], pts[qi, bi, 1]
                    bases[k, q] = [p0, p0 + X, p0 + X + Y, p0, p0 + X, p0 + X + Y,
                                   start_tri[qi, bi]]
            part.emit(lib, grp, gi, bases, points_t, total_points, conn_t, total_tris,
                      status_e + 8 * row, stream, dev)
            row += part.size * len(grp)

    if not copy_to_host:
        torch.cuda.current_stream(dev).synchronize()
    points_field = Field(f32, (total_points * 3,), CUDABuffer(points_t))
    conn_field = Field(i32, (total_tris * 3,), CUDABuffer(conn_t))
    points_h = conn_h = None
    if copy_to_host:
        # Page-locked destinations: the copies run at full link speed and
        # the returned numpy arrays keep their pinned blocks alive.
        points_h = torch.empty(points_t.shape, dtype=points_t.dtype, pin_memory=True)
        conn_h = torch.empty(conn_t.shape, dtype=conn_t.dtype, pin_memory=True)
        points_h.copy_(points_t, non_blocking=True)
        conn_h.copy_(conn_t, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    _raise_status(status_h.numpy()[nblk * niso:], "emit")
    out = {
        "points": points_h.numpy().reshape(-1, 3) if copy_to_host else None,
        "conn": conn_h.numpy().reshape(-1, 3) if copy_to_host else None,
        "points_field": points_field,
        "conn_field": conn_field,
        "total_points": total_points,
        "total_tris": total_tris,
        "block_point_counts": [int(x) for x in block_pts.sum(axis=0)],
        "block_tri_counts": [int(x) for x in tris.sum(axis=0)],
    }
    if is_list:
        out["isovalues"] = list(isos)
        out["isovalue_point_counts"] = [int(x) for x in block_pts.sum(axis=1)]
        out["isovalue_tri_counts"] = [int(x) for x in tris.sum(axis=1)]
    return out
