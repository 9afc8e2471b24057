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


def _torch_totals(v, shape, iso, num_tris, chunk=64):
    """Whole-volume totals {X, Y, Z, T} computed independently with torch:
    crossings as (s > iso) != (s' > iso) along each axis, triangles as
    num_tris[case] with the case built from the eight corners in the order
    of flying_edges.py:463-471 (0 (i,j,k), 1 (i+1,j,k), 2 (i+1,j+1,k),
    3 (i,j+1,k), 4-7 the same at k+1).  Processed in z-chunks."""
    nx1, ny1, nz1 = shape
    a = v.view(nz1, ny1, nx1)
    tab = torch.as_tensor(num_tris, dtype=torch.int64, device=v.device)
    X = Y = Z = T = 0
    for k0 in range(0, nz1, chunk):
        k1 = min(nz1, k0 + chunk + 1)  # one plane of overlap for z edges and cells
        b = a[k0:k1] > iso
        own = min(chunk, nz1 - k0)
        X += int((b[:own, :, 1:] != b[:own, :, :-1]).sum())
        Y += int((b[:own, 1:, :] != b[:own, :-1, :]).sum())
        if k1 - k0 > 1:
            Z += int((b[1:] != b[:-1]).sum())
            u = b.to(torch.uint8)
            c = (u[:-1, :-1, :-1] | (u[:-1, :-1, 1:] << 1) | (u[:-1, 1:, 1:] << 2) |
                 (u[:-1, 1:, :-1] << 3) | (u[1:, :-1, :-1] << 4) | (u[1:, :-1, 1:] << 5) |
                 (u[1:, 1:, 1:] << 6) | (u[1:, 1:, :-1] << 7))
            T += int(tab[c.long()].sum())
            del u, c
        del b
    return X, Y, Z, T


def _row_counts(rows, total):
    """Per-row counts from the library's exclusive section offsets."""
    return np.diff(np.append(rows, total))


def test_noise_2048_full_size(tack, oracle):
    """C5 at full size: 2048x2048x1024 nodes (16 GiB of f32), 4-octave value
    noise, isovalues -0.3, 0, 0.3, 0.6 in one pass.

    Checked (i) on the totals of every isovalue against an independent torch
    count over the whole volume, (ii) row by row against the oracle on three
    33-plane slabs (x, y, z crossings and triangles of every row there),
    (iii) exactly, points bit for bit, on one slab emitted as a volume of its
    own, and (iv) over the whole surface on the device: ids in range, every
    point referenced, no edge in more than two triangles, points inside the
    volume.
    """
    shape = (2048, 2048, 1024)
    isos = [-0.3, 0.0, 0.3, 0.6]
    v = workloads.generate("noise", shape)
    g = _grid(shape)
    nx, ny, nz = g[:3]
    got = capi_fe(v, g, isos, want_rows=True, host=False)
    counts = got["counts"]
    num_tris = oracle.tables()[1]
    # (i) whole-volume totals
    for q, iso in enumerate(isos):
        assert tuple(int(c) for c in counts[q]) == _torch_totals(v, shape, iso, num_tris), iso
    # (ii) every row of three slabs
    plane = shape[0] * shape[1]
    for k0 in (0, 496, 991):
        slab = v[k0 * plane:(k0 + 33) * plane].cpu().numpy()
        gs = (nx, ny, 32, 0.0, 0.0, float(k0), 1.0, 1.0, 1.0)
        for q, iso in enumerate(isos):
            info = oracle.count_block(slab, oracle.Grid(*gs), iso)
            rows = got["rows"][q]
            r0, r1 = k0 * (ny + 1), (k0 + 33) * (ny + 1)
            xc = _row_counts(rows[:, 0], counts[q][0])
            yc = _row_counts(rows[:, 1], counts[q][1])
            zc = _row_counts(rows[:, 2], counts[q][2])
            tc = _row_counts(rows[:, 3], counts[q][3]).reshape(nz + 1, ny + 1)[:nz, :ny]
            np.testing.assert_array_equal(xc[r0:r1], info["row_xc"])
            np.testing.assert_array_equal(yc[r0:r1], info["row_yc"])
            np.testing.assert_array_equal(zc[r0:r1 - (ny + 1)], info["row_zc"][:-(ny + 1)])
            np.testing.assert_array_equal(tc[k0:k0 + 32].reshape(-1), info["row_tri"])
        # (iii) the middle slab emitted on its own, exactly
        if k0 == 496:
            got_s = capi_fe(torch.from_numpy(slab).cuda(), gs, isos)
            ref_s = oracle.flying_edges_isovalues(slab, oracle.Grid(*gs), isos)
            assert_same_surface(got_s, ref_s)
            del got_s, ref_s
        del slab
    # (iv) whole-surface properties on the device
    P, T = got["total_points"], got["total_tris"]
    conn, pts = got["conn"], got["points"]
    assert int(conn.min()) >= 0 and int(conn.max()) < P
    used = torch.zeros(P, dtype=torch.bool, device=conn.device)
    used[conn.reshape(-1).long()] = True
    assert bool(used.all())
    del used
    assert bool(torch.isfinite(pts).all())
    lo = pts.amin(0).cpu().numpy()
    hi = pts.amax(0).cpu().numpy()
    assert (lo >= 0).all() and hi[0] <= nx and hi[1] <= ny and hi[2] <= nz
    keys = []
    for a, b in ((0, 1), (1, 2), (2, 0)):
        e0 = conn[:, a].long()
        e1 = conn[:, b].long()
        keys.append(torch.minimum(e0, e1) * (1 << 32) + torch.maximum(e0, e1))
    k = torch.cat(keys)
    del keys
    k, _ = torch.sort(k)
    assert not bool((k[2:] == k[:-2]).any())
    assert T == int(counts[:, 3].sum())
