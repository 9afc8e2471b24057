"""Z-slab sharded flying edges on the GPU.

On one GPU, every rank's slab is processed by its own SlabEngine in turn
(count with the ghost plane, bases from the stacked totals, emit with global
ids and the slab's plane offset) and the assembled result must equal the
oracle's single-volume output bit for bit.  With two or more GPUs the same
path runs under torchrun with NCCL (tests/slab_rank_main.py).
"""

import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from fe_helpers import assert_points_identical

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run_slabs_one_gpu(tack, vol_dev, grid, isos, world, bounds=None):
    from tack_b200.distributed import SlabEngine, SlabPlan, assemble, slab_bases
    nx, ny, nz = grid.nx, grid.ny, grid.nz
    plane = (nx + 1) * (ny + 1)
    plans = [SlabPlan(nz + 1, world, r, bounds=bounds) for r in range(world)]
    engines, counts, locals_ = [], [], []
    for p in plans:
        eng = SlabEngine(grid, p, isos)
        local = vol_dev[p.k0 * plane:p.k1 * plane]
        engines.append(eng)
        locals_.append(local)
        counts.append(eng.count(local))
    allc = np.stack(counts)
    parts = []
    for p, eng, local, c in zip(plans, engines, locals_, counts):
        b = slab_bases(allc, p.rank)
        pts, conn = eng.emit(local, c, b)
        eng.check()
        parts.append({"points": pts.cpu().numpy(), "conn": conn.cpu().numpy(), "counts": c,
                      "bases": b})
    return assemble(parts)


@pytest.mark.parametrize("shape,world", [((127, 95, 60), 2), ((127, 95, 60), 3),
                                         ((96, 70, 41), 4), ((40, 33, 17), 7)])
def test_slabs_match_single_volume_oracle(tack, oracle, shape, world):
    nx, ny, nz = shape
    rng = np.random.default_rng(nx * 31 + world)
    z, y, x = np.meshgrid(np.arange(nz + 1), np.arange(ny + 1), np.arange(nx + 1), indexing="ij")
    v = (np.sin(x * 0.21) * np.cos(y * 0.17) + np.sin(z * 0.13 + 0.4)
         + 0.2 * rng.standard_normal(x.shape)).astype(np.float32).reshape(-1)
    g = (nx, ny, nz, -1.25, 0.5, 2.0, 0.3, 0.45, 0.7)
    isos = [0.0, 0.6, -0.9]
    points, conn = _run_slabs_one_gpu(tack, torch.from_numpy(v).cuda(), tack.UniformGrid(*g),
                                      isos, world)
    ref = oracle.flying_edges_isovalues(v, oracle.Grid(*g), isos)
    np.testing.assert_array_equal(conn, ref["conn"])
    assert_points_identical(points, ref["points"])


def test_surface_balanced_slabs_match_single_volume(tack):
    """Slab bounds from the surface of a first pass (per-plane triangles from
    each equal slab's row table, a cost per node and per triangle): the
    slabs are uneven, and the sharded surface still equals the single-volume
    surface."""
    from tack_b200 import workloads
    from tack_b200.distributed import SlabEngine, SlabPlan, balanced_bounds
    shape = (128, 128, 128)
    whole = workloads.generate("blobs", shape)
    nx, ny, nz = shape[0] - 1, shape[1] - 1, shape[2] - 1
    grid = tack.UniformGrid(nx, ny, nz, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
    plane = shape[0] * shape[1]
    world = 4
    per_plane = []
    for r in range(world):
        p = SlabPlan(shape[2], world, r)
        eng = SlabEngine(grid, p, [0.5])
        local = whole[p.k0 * plane:p.k1 * plane]
        c = eng.count(local)
        per_plane.append(eng.plane_triangles(c))
    tris = np.concatenate(per_plane)
    assert tris.size == shape[2] and int(tris.sum()) > 0
    r = tack.flying_edges(tack.from_torch(whole), grid, 0.5)
    assert int(tris.sum()) == r["total_tris"]
    bounds = balanced_bounds(plane + 83.0 * tris, world)
    assert bounds != [0, 32, 64, 96, 128]
    points, conn = _run_slabs_one_gpu(tack, whole, grid, [0.5], world, bounds=bounds)
    np.testing.assert_array_equal(conn, r["conn"])
    assert_points_identical(points, r["points"])


def test_slabs_blobs_256_match_single_volume(tack):
    """A generated benchmark-style volume: slabs generated independently
    equal the planes of the whole volume, and the sharded surface equals the
    single-volume surface."""
    from tack_b200 import workloads
    shape = (256, 256, 256)
    whole = workloads.generate("blobs", shape)
    nx, ny, nz = shape[0] - 1, shape[1] - 1, shape[2] - 1
    grid = tack.UniformGrid(nx, ny, nz, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
    plane = shape[0] * shape[1]
    part = workloads.generate("blobs", shape, 100, 131)
    assert torch.equal(part, whole[100 * plane:131 * plane])
    points, conn = _run_slabs_one_gpu(tack, whole, grid, [0.5], 4)
    r = tack.flying_edges(tack.from_torch(whole), grid, 0.5)
    np.testing.assert_array_equal(conn, r["conn"])
    assert_points_identical(points, r["points"])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_torchrun_nccl(tmp_path):
    out = tmp_path / "slab2.txt"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=REPO)
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), os.path.join(REPO, "tests", "slab_rank_main.py"),
           str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=700)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert out.read_text().strip() == "ok"


def test_device_planned_emit_matches_host_planned(tack):
    """copy_counts -> plan -> emit_dev (bases in device memory) gives the same
    bytes as the host-planned emit, for every rank of a 3-way split, and a
    too-small output is reported, cleared and redone."""
    import ctypes
    from tack_b200 import _lib
    from tack_b200.distributed import SlabEngine, SlabPlan, slab_bases
    from fe_helpers import f32arr, stream
    lib = _lib.load()
    nx, ny, nz = 95, 70, 41
    rng = np.random.default_rng(7)
    z, y, x = np.meshgrid(np.arange(nz + 1), np.arange(ny + 1), np.arange(nx + 1), indexing="ij")
    v = (np.sin(x * 0.2) + np.cos(y * 0.15 + z * 0.1) + 0.1 * rng.standard_normal(x.shape))
    vol = torch.from_numpy(v.astype(np.float32).reshape(-1)).cuda()
    g = tack.UniformGrid(nx, ny, nz, 0.5, 1.0, -2.0, 0.25, 0.5, 0.75)
    isos = [0.0, 0.7]
    world, niso = 3, len(isos)
    plane = (nx + 1) * (ny + 1)
    plans = [SlabPlan(nz + 1, world, r) for r in range(world)]
    engs = [SlabEngine(g, p, isos) for p in plans]
    slabs = [vol[p.k0 * plane:p.k1 * plane] for p in plans]
    counts = [e.count(sv) for e, sv in zip(engs, slabs)]
    allc = np.stack(counts)
    gathered = torch.zeros(world * niso * 4, dtype=torch.int64, device="cuda")
    st = stream()
    for r, e in enumerate(engs):
        dst = gathered[r * niso * 4:(r + 1) * niso * 4]
        assert lib.tkmc_fe_copy_counts(nx, ny, plans[r].nz_cells, niso, e.ws.data_ptr(),
                                       e.nbytes, dst.data_ptr(), st) == 0
    geom = f32arr([g.x0, g.y0, g.z0, g.dx, g.dy, g.dz])
    for r, (p, e, sv) in enumerate(zip(plans, engs, slabs)):
        b = slab_bases(allc, r)
        want_p, want_c = e.emit(sv, counts[r], b)
        bases = torch.zeros(niso * 7, dtype=torch.int64, device="cuda")
        assert lib.tkmc_fe_plan(gathered.data_ptr(), world, r, niso, 0, bases.data_ptr(), st) == 0
        host_b = np.concatenate([b["id_base"], b["out_base"], b["tri_out"][:, None]], axis=1)
        np.testing.assert_array_equal(bases.cpu().numpy().reshape(niso, 7), host_b)
        P, T = int(counts[r][:, :3].sum()), int(counts[r][:, 3].sum())
        ghost = 1 if p.ghost else 0
        # Too small first: the emit skips what does not fit and reports it.
        small_p = torch.empty(3 * max(P // 2, 1), dtype=torch.float32, device="cuda")
        small_c = torch.empty(3 * max(T // 2, 1), dtype=torch.int32, device="cuda")
        args = (sv.data_ptr(), nx, ny, p.nz_cells, ghost, p.k0, geom, f32arr(isos), niso, None,
                e.ws.data_ptr(), e.nbytes, bases.data_ptr())
        assert lib.tkmc_fe_emit_dev(*args, small_p.data_ptr(), small_p.numel() // 3,
                                    small_c.data_ptr(), small_c.numel() // 3, st) == 0
        assert lib.tkmc_fe_check(nx, ny, p.nz_cells, niso, e.ws.data_ptr(), e.nbytes,
                                 st) == _lib.TKMC_ERR_CAPACITY
        assert lib.tkmc_fe_clear_capacity_error(nx, ny, p.nz_cells, niso, e.ws.data_ptr(),
                                                e.nbytes, st) == 0
        pts = torch.empty(3 * P, dtype=torch.float32, device="cuda")
        cn = torch.empty(3 * T, dtype=torch.int32, device="cuda")
        assert lib.tkmc_fe_emit_dev(*args, pts.data_ptr(), P, cn.data_ptr(), T, st) == 0
        assert lib.tkmc_fe_check(nx, ny, p.nz_cells, niso, e.ws.data_ptr(), e.nbytes, st) == 0
        assert torch.equal(pts.view(torch.int32), want_p.view(torch.int32))
        assert torch.equal(cn, want_c)
    del ctypes


def test_run_device_single_volume(tack):
    """SlabEngine.run_device on one GPU (world 1) equals the host-planned run."""
    from tack_b200 import workloads
    from tack_b200.distributed import SlabEngine, SlabPlan
    shape = (128, 96, 80)
    vol = workloads.generate("blobs", shape)
    g = tack.UniformGrid(shape[0] - 1, shape[1] - 1, shape[2] - 1, 0, 0, 0, 1, 1, 1)
    eng = SlabEngine(g, SlabPlan(shape[2], 1, 0), [0.5, 0.9])
    ref = eng.run(vol)
    P = int(ref["counts"][:, :3].sum())
    T = int(ref["counts"][:, 3].sum())
    pts = torch.empty(3 * P, dtype=torch.float32, device="cuda")
    cn = torch.empty(3 * T, dtype=torch.int32, device="cuda")
    counts_host = torch.zeros(8, dtype=torch.int64, pin_memory=True)
    for _ in range(2):
        eng.run_device(vol, pts, cn, counts_host)
    eng.check()
    np.testing.assert_array_equal(counts_host.numpy().reshape(2, 4), ref["counts"])
    assert torch.equal(pts.view(torch.int32), ref["points_field"].tensor.view(torch.int32))
    assert torch.equal(cn, ref["conn_field"].tensor)


def test_graph_replay_single_volume(tack):
    """The device-planned step captured in a CUDA graph: each replay rewrites
    the same bytes as the host-planned run."""
    from tack_b200 import workloads
    from tack_b200.distributed import SlabEngine, SlabPlan
    shape = (160, 96, 64)
    vol = workloads.generate("gyroid", shape)
    g = tack.UniformGrid(shape[0] - 1, shape[1] - 1, shape[2] - 1, 0, 0, 0, 1, 1, 1)
    eng = SlabEngine(g, SlabPlan(shape[2], 1, 0), [0.0])
    ref = eng.run(vol)
    P = int(ref["counts"][:, :3].sum())
    T = int(ref["counts"][:, 3].sum())
    pts = torch.empty(3 * P, dtype=torch.float32, device="cuda")
    cn = torch.empty(3 * T, dtype=torch.int32, device="cuda")
    counts_host = torch.zeros(4, dtype=torch.int64, pin_memory=True)
    graph = eng.capture(vol, pts, cn, counts_host)
    for _ in range(3):
        pts.zero_()
        cn.zero_()
        counts_host.zero_()
        graph.replay()
        torch.cuda.synchronize()
        eng.check()
        np.testing.assert_array_equal(counts_host.numpy().reshape(1, 4), ref["counts"])
        assert torch.equal(pts.view(torch.int32), ref["points_field"].tensor.view(torch.int32))
        assert torch.equal(cn, ref["conn_field"].tensor)
    del graph


def test_shared_output_plan_single_gpu_parts(tack, oracle):
    """Several z-parts on one GPU planned with shared_output=1 write one
    output in the single-volume layout: equal to the oracle's surface."""
    from tack_b200 import _lib
    from tack_b200.distributed import SlabEngine, SlabPlan
    from fe_helpers import f32arr, stream
    lib = _lib.load()
    nx, ny, nz = 127, 40, 50
    rng = np.random.default_rng(3)
    z, y, x = np.meshgrid(np.arange(nz + 1), np.arange(ny + 1), np.arange(nx + 1), indexing="ij")
    v = (np.cos(x * 0.1) * np.sin(y * 0.2) + np.sin(z * 0.15)
         + 0.05 * rng.standard_normal(x.shape)).astype(np.float32).reshape(-1)
    vol = torch.from_numpy(v).cuda()
    g = tack.UniformGrid(nx, ny, nz, 1.0, 2.0, 3.0, 0.5, 0.5, 0.5)
    isos = [0.1, -0.4]
    parts, niso = 4, len(isos)
    plane = (nx + 1) * (ny + 1)
    plans = [SlabPlan(nz + 1, parts, r) for r in range(parts)]
    engs = [SlabEngine(g, p, isos) for p in plans]
    slabs = [vol[p.k0 * plane:p.k1 * plane] for p in plans]
    counts = np.stack([e.count(sv) for e, sv in zip(engs, slabs)])
    P, T = int(counts[:, :, :3].sum()), int(counts[:, :, 3].sum())
    dev_counts = torch.from_numpy(counts.reshape(-1).copy()).cuda()
    pts = torch.zeros(3 * P, dtype=torch.float32, device="cuda")
    cn = torch.zeros(3 * T, dtype=torch.int32, device="cuda")
    geom = f32arr([g.x0, g.y0, g.z0, g.dx, g.dy, g.dz])
    st = stream()
    for r, (p, e, sv) in enumerate(zip(plans, engs, slabs)):
        bases = torch.zeros(niso * 7, dtype=torch.int64, device="cuda")
        assert lib.tkmc_fe_plan(dev_counts.data_ptr(), parts, r, niso, 1, bases.data_ptr(), st) == 0
        assert lib.tkmc_fe_emit_dev(sv.data_ptr(), nx, ny, p.nz_cells, 1 if p.ghost else 0, p.k0,
                                    geom, f32arr(isos), niso, None, e.ws.data_ptr(), e.nbytes,
                                    bases.data_ptr(), pts.data_ptr(), P, cn.data_ptr(), T,
                                    st) == 0
        assert lib.tkmc_fe_check(nx, ny, p.nz_cells, niso, e.ws.data_ptr(), e.nbytes, st) == 0
    ref = oracle.flying_edges_isovalues(v, oracle.Grid(nx, ny, nz, g.x0, g.y0, g.z0, g.dx, g.dy,
                                                       g.dz), isos)
    np.testing.assert_array_equal(cn.cpu().numpy().reshape(-1, 3), ref["conn"])
    assert_points_identical(pts.cpu().numpy().reshape(-1, 3), ref["points"])


@pytest.mark.parametrize("cells", [(127, 70, 41), (95, 70, 41), (255, 300, 9),
                                   (127, 255, 200)])
def test_exchange_after_count_pass_plans_like_host(tack, cells):
    """The peer exchange launched right after the count pass (its totals
    summed from the tile totals and the row counts of a partial tile, since
    the ghost plane's rows are excluded) plans the same bases as the host
    from the full count, while the offsets pass runs on the main stream;
    then the emit equals the host-planned emit.  One rank (world 1), so the
    exchange waits only for itself; rows of 128 and 256 nodes take the
    tile-total path, rows of 96 nodes the row-scan path."""
    import ctypes
    from tack_b200 import _lib
    from tack_b200.distributed import SlabEngine, SlabPlan, slab_bases
    from fe_helpers import f32arr, stream
    lib = _lib.load()
    nx, ny, nz = cells
    rng = np.random.default_rng(nx + ny)
    z, y, x = np.meshgrid(np.arange(nz + 1), np.arange(ny + 1), np.arange(nx + 1), indexing="ij")
    v = (np.sin(x * 0.11) * np.cos(y * 0.07) + np.sin(z * 0.3 + 0.2)
         + 0.1 * rng.standard_normal(x.shape)).astype(np.float32).reshape(-1)
    vol = torch.from_numpy(v).cuda()
    g = tack.UniformGrid(nx, ny, nz, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
    isos = [0.0, 0.5, -0.6]
    niso = len(isos)
    plane = (nx + 1) * (ny + 1)
    # Rank 0 of a two-way split: its slab has a ghost plane.
    p = SlabPlan(nz + 1, 2, 0)
    e = SlabEngine(g, p, isos)
    sv = vol[p.k0 * plane:p.k1 * plane]
    counts = e.count(sv)
    want_p, want_c = e.emit(sv, counts, slab_bases(counts[None], 0))
    x = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(lib.tkmc_exchange_handle_bytes())
    _lib.check(lib.tkmc_exchange_create(1, 0, niso, ctypes.byref(x), handle), "create")
    try:
        members = (ctypes.c_void_p * 1)(x.value)
        _lib.check(lib.tkmc_exchange_connect_local(x, members), "connect_local")
        bases = torch.full((niso * 7,), -5, dtype=torch.int64, device="cuda")
        side = torch.cuda.Stream()
        main = torch.cuda.current_stream()
        for _ in range(2):  # two epochs
            bases.fill_(-5)
            _lib.check(lib.tkmc_fe_classify(sv.data_ptr(), nx, ny, p.nz_cells, f32arr(isos), niso,
                                            e.ws.data_ptr(), e.nbytes, stream()), "classify")
            _lib.check(lib.tkmc_fe_scan_part(nx, ny, p.nz_cells, 1, niso, None, e.ws.data_ptr(),
                                             e.nbytes, 1, stream()), "scan part 1")
            side.wait_stream(main)
            _lib.check(lib.tkmc_exchange_plan_counts(x, nx, ny, p.nz_cells, 1, e.ws.data_ptr(),
                                                     e.nbytes, 0, bases.data_ptr(),
                                                     side.cuda_stream), "plan_counts")
            _lib.check(lib.tkmc_fe_scan_part(nx, ny, p.nz_cells, 1, niso, None, e.ws.data_ptr(),
                                             e.nbytes, 2, stream()), "scan part 2")
            main.wait_stream(side)
            b = slab_bases(counts[None], 0)
            host_b = np.concatenate([b["id_base"], b["out_base"], b["tri_out"][:, None]], axis=1)
            np.testing.assert_array_equal(bases.cpu().numpy().reshape(niso, 7), host_b)
            P, T = int(counts[:, :3].sum()), int(counts[:, 3].sum())
            pts = torch.empty(3 * P, dtype=torch.float32, device="cuda")
            cn = torch.empty(3 * T, dtype=torch.int32, device="cuda")
            _lib.check(lib.tkmc_fe_emit_dev(sv.data_ptr(), nx, ny, p.nz_cells, 1, p.k0,
                                            f32arr([0, 0, 0, 1, 1, 1]), f32arr(isos), niso, None,
                                            e.ws.data_ptr(), e.nbytes, bases.data_ptr(),
                                            pts.data_ptr(), P, cn.data_ptr(), T, stream()),
                       "emit_dev")
            _lib.check(lib.tkmc_fe_check(nx, ny, p.nz_cells, niso, e.ws.data_ptr(), e.nbytes,
                                         stream()), "check")
            assert torch.equal(pts.view(torch.int32), want_p.view(torch.int32))
            assert torch.equal(cn, want_c)
        assert lib.tkmc_fe_scan_part(nx, ny, p.nz_cells, 1, niso, None, e.ws.data_ptr(), e.nbytes,
                                     3, stream()) == _lib.TKMC_ERR_INVALID_ARG
    finally:
        torch.cuda.synchronize()
        lib.tkmc_exchange_destroy(x)
