"""Smooth vertex normals of a triangle mesh on sm_100a.

Drop-in for packages/tack-vis/src/tack/algorithms/compute_normals.py:
``compute_normals(points, conn, n_pts, n_tris)`` returns an f32 field of
n_pts * 3 interleaved normals: every triangle's area-weighted face normal
cross(v1 - v0, v2 - v0) added to its three vertices, then each vertex sum
longer than 1e-10 normalised.

The sums are 64-bit fixed point (tkmc_compute_normals), so the result is
the same on every run; the reference adds f32 atomics in whatever order the
threads run.  Against the reference's serial order the normals agree to
float rounding (tests: 1e-6 on unit normals away from cancellation).
"""

import torch

from .. import _lib
from ..field import CUDABuffer, Field, device_tensor, f32, i32
from ..runtime import current_device, current_stream, workspace

__all__ = ["compute_normals"]


def compute_normals(points, conn, n_pts, n_tris):
    """Vertex normals.

    Args:
        points: f32 field of at least n_pts*3 interleaved coordinates (a
            tack_b200 Field, a torch tensor, a reference CUDA field, or a
            host array).
        conn: int32 field of at least n_tris*3 point ids in [0, n_pts).
        n_pts, n_tris: numbers of points and triangles.

    Returns:
        Field f32 (n_pts*3,), interleaved normals.
    """
    n_pts, n_tris = int(n_pts), int(n_tris)
    if n_pts < 0 or n_tris < 0:
        raise ValueError("n_pts and n_tris must be >= 0")
    p = device_tensor(points, f32)
    c = device_tensor(conn, i32)
    if p.numel() < 3 * n_pts or c.numel() < 3 * n_tris:
        raise ValueError(f"points hold {p.numel() // 3} points and conn {c.numel() // 3} "
                         f"triangles; {n_pts} and {n_tris} were asked for")
    dev = current_device()
    lib = _lib.load()
    out = torch.empty(max(3 * n_pts, 1), dtype=torch.float32, device=dev)
    nbytes = lib.tkmc_normals_workspace_bytes(n_pts)
    ws = workspace("normals", nbytes, dev)
    _lib.check(lib.tkmc_compute_normals(p.data_ptr(), c.data_ptr(), n_pts, n_tris, ws.data_ptr(),
                                        ws.numel(), out.data_ptr(), current_stream(dev)),
               "tkmc_compute_normals")
    return Field(f32, (3 * n_pts,), CUDABuffer(out[:3 * n_pts]))
