"""Vertex normals on the GPU against the reference's (compute_normals.py).

The library adds face normals in 64-bit fixed point, the reference in f32
(serially on its CPU backend, by atomics on a GPU), so they agree to f32
rounding of the sums: the test allows 2e-6 on a unit normal, scaled up where
a vertex's faces nearly cancel (the sum of the face-normal lengths over the
length of their sum).  Zero sums are exact, and repeated calls give the same
bits.
"""

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _gpu_normals(tack, points, conn):
    p = torch.from_numpy(np.ascontiguousarray(points, np.float32).reshape(-1)).cuda()
    c = torch.from_numpy(np.ascontiguousarray(conn, np.int32).reshape(-1)).cuda()
    out = tack.compute_normals(p, c, points.shape[0], conn.shape[0])
    return out.to_numpy().reshape(-1, 3)


def _tolerance(points, conn):
    """Per-vertex allowed error: 2e-6 times the cancellation of its faces."""
    p = points.astype(np.float64)
    e1 = p[conn[:, 1]] - p[conn[:, 0]]
    e2 = p[conn[:, 2]] - p[conn[:, 0]]
    fn = np.cross(e1, e2)
    s = np.zeros(points.shape[0])
    a = np.zeros((points.shape[0], 3))
    for v in range(3):
        np.add.at(s, conn[:, v], np.linalg.norm(fn, axis=1))
        np.add.at(a, conn[:, v], fn)
    ratio = np.where(np.linalg.norm(a, axis=1) > 0, s / np.maximum(np.linalg.norm(a, axis=1), 1e-300),
                     1.0)
    return 2e-6 * np.maximum(ratio, 1.0)[:, None]


def _cases():
    z = np.load(f"{GOLDEN}/normals.npz")
    names = sorted({k.rsplit("_", 1)[0] for k in z.files})
    return [(n, z[f"{n}_points"], z[f"{n}_conn"], z[f"{n}_normals"]) for n in names]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0])
def test_normals_match_reference(tack, case):
    name, points, conn, ref = case
    got = _gpu_normals(tack, points, conn)
    assert np.all(np.abs(got - ref) <= _tolerance(points, conn)), name
    zero = np.all(ref == 0, axis=1)
    np.testing.assert_array_equal(got[zero], 0.0)


def test_normals_are_deterministic(tack):
    z = np.load(f"{GOLDEN}/normals.npz")
    p, c = z["random_points"], z["random_conn"]
    a = _gpu_normals(tack, p, c)
    for _ in range(3):
        np.testing.assert_array_equal(_gpu_normals(tack, p, c).view(np.uint32), a.view(np.uint32))


def test_isosurface_normals_match_oracle(tack, oracle):
    """The flying-edges surface of a generated volume, straight from device
    fields, as a pipeline would call it."""
    from tack_b200 import workloads
    shape = (192, 160, 128)
    vol = workloads.generate("gyroid", shape)
    g = tack.UniformGrid(shape[0] - 1, shape[1] - 1, shape[2] - 1, -1.0, -1.0, -1.0, 0.01, 0.01, 0.01)
    r = tack.flying_edges(tack.from_torch(vol), g, 0.0)
    n = tack.compute_normals(r["points_field"], r["conn_field"], r["total_points"],
                             r["total_tris"]).to_numpy().reshape(-1, 3)
    ref = oracle.compute_normals(r["points"], r["conn"])
    assert np.all(np.abs(n - ref) <= _tolerance(r["points"], r["conn"]))
    np.testing.assert_allclose(np.linalg.norm(n, axis=1), 1.0, atol=1e-5)


def test_bad_ids_and_nan_points(tack):
    p = np.array([[0, 0, 0], [1, 0, 0], [0, 1, 0], [np.nan, 0, 0], [1, 1, 0]], np.float32)
    with pytest.raises(RuntimeError, match="point id"):
        _gpu_normals(tack, p, np.array([[0, 1, 7]], np.int32))
    got = _gpu_normals(tack, p, np.array([[0, 1, 2], [1, 3, 4]], np.int32))
    assert np.isnan(got[[1, 3, 4]]).all()  # every vertex of the face with a NaN corner
    np.testing.assert_allclose(got[[0, 2]], [[0, 0, 1], [0, 0, 1]], atol=1e-6)
    empty = tack.compute_normals(torch.zeros(0, device="cuda"),
                                 torch.zeros(0, dtype=torch.int32, device="cuda"), 0, 0)
    assert empty.shape == (0,)
