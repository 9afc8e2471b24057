"""Per-cell marching-cubes classification on sm_100a.

The per-cell form of packages/tack-vis/examples/26_marching_cubes.py:435-450
(``classify_cells``): for every cell its 8-corner case index (bit b set when
corner b is above the isovalue, strict ``>``) and its triangle count.
Together with ``exclusive_scan`` this gives the example's per-cell offsets.
"""

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
