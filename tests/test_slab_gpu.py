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


def _run_slabs_one_gpu(tack, vol_dev, grid, isos, world):
    from tack_b200.distributed import SlabEngine, SlabPlan, assemble, slab_bases
    nx, ny, nz = grid.nx, grid.ny, grid.nz
    plane = (nx + 1) * (ny + 1)
    plans = [SlabPlan(nz + 1, world, r) for r in range(world)]
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
