"""The benchmark configurations on the GPU, against the oracle.

Volumes are generated on the GPU (tack_b200.workloads) and copied to the
host, so both sides read the same bytes.  Sizes up to 512^3 are compared in
full (counts, offsets, connectivity exact; points bit-exact); the 1024^3
headline volume is compared on its counts and offsets in full and on the
emitted surface through size-independent properties plus an exact slab.
"""

import numpy as np
import pytest
import torch

from fe_helpers import assert_same_surface, capi_fe, reference_offsets_from_rows
from tack_b200 import workloads

pytestmark = pytest.mark.gpu


def _grid(shape):
    nx, ny, nz = shape
    return (nx - 1, ny - 1, nz - 1, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)


@pytest.mark.parametrize("name,shape,isos", [
    ("sphere", (64, 64, 64), [0.0]),
    ("gyroid", (256, 256, 256), [0.0]),
    ("sines", (256, 256, 256), [0.25]),
    ("blobs", (256, 256, 256), [0.5]),
    ("noise", (256, 256, 128), [-0.3, 0.0, 0.3, 0.6]),
    ("sines", (512, 512, 512), [0.25]),
])
def test_config_matches_oracle(tack, oracle, name, shape, isos):
    v = workloads.generate(name, shape)
    g = _grid(shape)
    got = capi_fe(v, g, isos, want_rows=True)
    host = v.cpu().numpy()
    ref = oracle.flying_edges_isovalues(host, oracle.Grid(*g), isos)
    assert_same_surface(got, ref)
    for q, iso in enumerate(isos):
        info = oracle.count_block(host, oracle.Grid(*g), iso)
        xo, yo, zo, to = reference_offsets_from_rows(got["rows"][q], got["counts"][q], g)
        np.testing.assert_array_equal(xo, info["xo"])
        np.testing.assert_array_equal(yo, info["yo"])
        np.testing.assert_array_equal(zo, info["zo"])
        np.testing.assert_array_equal(to, info["tri_offsets"])


def test_sphere_config_is_reference_c1(tack):
    """The generated C1 volume is byte-identical to the reference fixture."""
    from conftest import load_fe_case
    c = load_fe_case("c1_sphere64")
    v = workloads.generate("sphere").cpu().numpy()
    np.testing.assert_array_equal(v.view(np.uint32), c["values"].view(np.uint32))


def test_blobs_1024_headline(tack, oracle):
    """C4 (1024^3, 32 Gaussian blobs, isovalue 0.5).

    Counts and every row offset are compared with the oracle over the whole
    volume; the emitted surface is checked exactly on a 64-plane slab and
    through properties over the whole volume: conn ids in range, every point
    referenced, every interior edge shared by exactly two triangles.
    """
    shape = (1024, 1024, 1024)
    v = workloads.generate("blobs", shape)
    g = _grid(shape)
    got = capi_fe(v, g, [0.5], want_rows=True)
    host = v.cpu().numpy()
    info = oracle.count_block(host, oracle.Grid(*g), 0.5)
    xo, yo, zo, to = reference_offsets_from_rows(got["rows"][0], got["counts"][0], g)
    np.testing.assert_array_equal(xo, info["xo"])
    np.testing.assert_array_equal(yo, info["yo"])
    np.testing.assert_array_equal(zo, info["zo"])
    np.testing.assert_array_equal(to, info["tri_offsets"])
    assert got["total_points"] == info["total_points"]
    assert got["total_tris"] == info["total_tris"]
    conn = got["conn"]
    assert conn.min() >= 0 and conn.max() < got["total_points"]
    assert np.unique(conn).size == got["total_points"]
    # Interior edges (not on the volume boundary) are shared by two triangles.
    e = np.concatenate([conn[:, [0, 1]], conn[:, [1, 2]], conn[:, [2, 0]]])
    e.sort(axis=1)
    key = e[:, 0].astype(np.int64) * (1 << 32) + e[:, 1]
    _, cnt = np.unique(key, return_counts=True)
    assert set(np.unique(cnt)) <= {1, 2}
    # Exact comparison on a slab: planes 480..544 as a volume of its own.
    k0, k1 = 480, 545
    slab = host.reshape(1024, 1024, 1024)[k0:k1].reshape(-1)
    gs = (1023, 1023, k1 - k0 - 1, 0.0, 0.0, float(k0), 1.0, 1.0, 1.0)
    got_s = capi_fe(torch.from_numpy(slab).cuda(), gs, [0.5])
    ref_s = oracle.flying_edges(slab, oracle.Grid(*gs), 0.5)
    assert_same_surface(got_s, ref_s)
