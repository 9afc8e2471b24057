"""Per-cell marching cubes on sm_100a: classification and the unmerged
triangle soup.

``classify_cells`` is the per-cell form of
packages/tack-vis/examples/26_marching_cubes.py:435-450: for every cell its
8-corner case index (bit b set when corner b is above the isovalue, strict
``>``) and its triangle count; with ``exclusive_scan`` this gives the
example's per-cell offsets.  ``marching_cubes_soup`` is the example's whole
pipeline (classify_cells, exclusive_scan, emit_triangles, :435-503): every
triangle's three vertices written out on their own, SoA x/y/z, bit-identical
to emit_triangles -- for renderers that want no index buffer.
"""

import ctypes

import numpy as np
import torch

from .. import _lib
from ..field import CUDABuffer, Field, device_tensor, f32, i32, u8
from ..runtime import current_device, current_stream, workspace


def classify_cells(scalar, grid, isovalue, mask=None):
    """Return (cases, num_tri) fields: u8 case index and i32 triangle count
    per cell (cells in i-fastest order, nx*ny*nz of them).  Masked cells
    (mask != 0) get 0 triangles."""
    v = device_tensor(scalar, f32)
    g = grid
    if v.numel() != (g.nx + 1) * (g.ny + 1) * (g.nz + 1):
        raise ValueError("field size does not match the grid")
    m = None if mask is None else device_tensor(mask, i32)
    ncell = g.nx * g.ny * g.nz
    dev = current_device()
    cases = torch.empty(ncell, dtype=torch.uint8, device=dev)
    ntri = torch.empty(ncell, dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws = workspace("fe", lib.tkmc_fe_workspace_bytes(g.nx, g.ny, g.nz, 1), dev)
    _lib.check(lib.tkmc_mc_classify_cells(
        v.data_ptr(), g.nx, g.ny, g.nz, float(isovalue), m.data_ptr() if m is not None else None,
        ws.data_ptr(), ws.numel(), cases.data_ptr(), ntri.data_ptr(), current_stream(dev)),
        "tkmc_mc_classify_cells")
    return (Field(u8, (ncell,), CUDABuffer(cases)), Field(i32, (ncell,), CUDABuffer(ntri)))


def marching_cubes_soup(scalar, grid, isovalue, mask=None, *, copy_to_host=True):
    """The unmerged triangle soup of a uniform grid.

    Args:
        scalar: f32 field of (nx+1)*(ny+1)*(nz+1) node values, i fastest.
        grid: UniformGrid (nx, ny, nz cells, origin, spacing).
        isovalue: threshold, or a sequence of up to 8 thresholds (each
            isovalue's triangles follow the previous one's).
        mask: optional int32 per cell; masked cells emit nothing.

    Returns:
        dict with 'x', 'y', 'z' (numpy f32 (3*T,): vertex v of triangle t at
        3t+v; None when copy_to_host=False), 'x_field', 'y_field', 'z_field'
        (device fields), 'total_tris' and, for a sequence of isovalues,
        'isovalue_tri_counts'; None when there are no triangles.
    """
    is_list = not np.isscalar(isovalue) and not isinstance(isovalue, (float, int))
    isos = [float(x) for x in (isovalue if is_list else [isovalue])]
    if not 1 <= len(isos) <= _lib.MAX_ISO:
        raise ValueError(f"1 to {_lib.MAX_ISO} isovalues per call")
    v = device_tensor(scalar, f32)
    g = grid
    if v.numel() != (g.nx + 1) * (g.ny + 1) * (g.nz + 1):
        raise ValueError("field size does not match the grid")
    m = None if mask is None else device_tensor(mask, i32)
    if m is not None and m.numel() != g.nx * g.ny * g.nz:
        raise ValueError("mask size does not match the grid")
    dev = current_device()
    st = current_stream(dev)
    lib = _lib.load()
    niso = len(isos)
    nbytes = lib.tkmc_fe_workspace_bytes(g.nx, g.ny, g.nz, niso)
    if nbytes == 0:
        raise ValueError(f"unsupported grid {g.nx} x {g.ny} x {g.nz}")
    ws = workspace("fe", nbytes, dev)
    isoc = (ctypes.c_float * niso)(*isos)
    mptr = m.data_ptr() if m is not None else None
    counts = np.zeros(niso * 4, np.int64)
    _lib.check(lib.tkmc_fe_count(v.data_ptr(), g.nx, g.ny, g.nz, 0, isoc, niso, mptr,
                                 ws.data_ptr(), ws.numel(), counts.ctypes.data, st),
               "tkmc_fe_count")
    tris = counts.reshape(niso, 4)[:, 3]
    total = int(tris.sum())
    if total == 0:
        return None
    base = np.concatenate([[0], np.cumsum(tris)[:-1]]).astype(np.int64)
    outs = [torch.empty(3 * total, dtype=torch.float32, device=dev) for _ in range(3)]
    geom = (ctypes.c_float * 6)(g.x0, g.y0, g.z0, g.dx, g.dy, g.dz)
    _lib.check(lib.tkmc_fe_emit_soup(v.data_ptr(), g.nx, g.ny, g.nz, geom, isoc, niso, mptr,
                                     ws.data_ptr(), ws.numel(), base.ctypes.data,
                                     outs[0].data_ptr(), outs[1].data_ptr(), outs[2].data_ptr(),
                                     total, st), "tkmc_fe_emit_soup")
    _lib.check(lib.tkmc_fe_check(g.nx, g.ny, g.nz, niso, ws.data_ptr(), ws.numel(), st),
               "tkmc_fe_check")
    fields = [Field(f32, (3 * total,), CUDABuffer(o)) for o in outs]
    out = {"x_field": fields[0], "y_field": fields[1], "z_field": fields[2],
           "total_tris": total,
           "x": outs[0].cpu().numpy() if copy_to_host else None,
           "y": outs[1].cpu().numpy() if copy_to_host else None,
           "z": outs[2].cpu().numpy() if copy_to_host else None}
    if is_list:
        out["isovalue_tri_counts"] = [int(t) for t in tris]
    return out
