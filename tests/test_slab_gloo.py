"""Z-slab sharding host logic on CPU: plans, the totals all-gather over a
gloo process group, global bases and assembly.

The per-rank kernels are stood in for by the oracle run on each rank's local
slab (own planes + one ghost plane), with its local point ids mapped to
global ids the way tkmc_fe_emit maps them from the bases (ghost-plane x/y
points continue past the rank's own totals into the next rank's range).  The
assembled result must equal the oracle's single-volume output bit for bit.
The GPU side of the same path is tested in test_slab_gpu.py.
"""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from tack_b200.distributed import (SlabPlan, assemble, balanced_bounds, gather_counts,
                                   rebalanced_bounds, slab_bases)

SHAPE = (23, 17, 29)          # cells; node planes along z: 30


def _volume(seed=3):
    nx, ny, nz = SHAPE
    rng = np.random.default_rng(seed)
    z, y, x = np.meshgrid(np.arange(nz + 1), np.arange(ny + 1), np.arange(nx + 1), indexing="ij")
    v = np.sqrt((x - 11.3) ** 2 + (y - 8.1) ** 2 + (z - 14.7) ** 2) - 9.0
    v = v + 0.4 * rng.standard_normal(v.shape)
    return v.astype(np.float32)


def _grid_args(k0=0):
    # z0 = 0, dz = 1: a node's z is float(k) whether computed globally or
    # from a local grid starting at plane k0, so the oracle on a slab gives
    # the same bits as the kernel's float(k + k_offset).
    nx, ny, nz = SHAPE
    return (nx, ny, nz, 0.5, -2.0, float(k0), 0.25, 0.75, 1.0)


def _rank_counts(oracle, vol, plan, isos):
    """Per isovalue {X, Y, Z, T} owned by this rank, plus the oracle's block
    info for the local slab."""
    nx, ny, _ = SHAPE
    local = vol[plan.k0:plan.k1]
    g = oracle.Grid(nx, ny, plan.nz_cells, *_grid_args(plan.k0)[3:])
    own_rows = (ny + 1) * (plan.p1 - plan.p0)
    counts, infos = [], []
    for iso in isos:
        info = oracle.count_block(local, g, iso)
        own_x = int(info["row_xc"][:own_rows].sum())
        own_y = int(info["row_yc"][:own_rows].sum())
        counts.append([own_x, own_y, info["total_z"], info["total_tris"]])
        infos.append(info)
    return np.array(counts, np.int64), infos, local, g


def _rank_emit(oracle, local, g, isos, infos, counts, bases):
    """Rank-local slices of the global output, laid out as tkmc_fe_emit
    lays them out (out_base, tri_out) with global point ids (id_base)."""
    own_p = int(counts[:, :3].sum())
    own_t = int(counts[:, 3].sum())
    pts = np.zeros((own_p, 3), np.float32)
    conn = np.zeros((own_t, 3), np.int32)
    for q, (iso, info) in enumerate(zip(isos, infos)):
        P, T = info["total_points"], info["total_tris"]
        lp = np.zeros(P * 3, np.float32)
        lc = np.zeros(T * 3, np.int32)
        if P or T:
            oracle.emit_block(local, g, iso, info, 0, 0, lp, lc)
        lp = lp.reshape(-1, 3)
        lx, ly = info["total_x"], info["total_y"]
        sect = [(0, counts[q, 0]), (lx, counts[q, 1]), (lx + ly, counts[q, 2])]
        for s, (lo, n) in enumerate(sect):
            ob = int(bases["out_base"][q, s])
            pts[ob:ob + n] = lp[lo:lo + n]
        lc = lc.reshape(-1, 3).astype(np.int64)
        gid = np.where(lc < lx, bases["id_base"][q, 0] + lc,
                       np.where(lc < lx + ly, bases["id_base"][q, 1] + (lc - lx),
                                bases["id_base"][q, 2] + (lc - lx - ly)))
        tb = int(bases["tri_out"][q])
        conn[tb:tb + T] = gid
    return {"points": pts.reshape(-1), "conn": conn.reshape(-1), "counts": counts,
            "bases": bases}


def _reference(oracle, vol, isos):
    nx, ny, nz = SHAPE
    return oracle.flying_edges_isovalues(vol, oracle.Grid(*_grid_args()), isos)


def _check(parts, ref):
    points, conn = assemble(parts)
    assert points.shape == ref["points"].shape and conn.shape == ref["conn"].shape
    np.testing.assert_array_equal(points.view(np.uint32), ref["points"].view(np.uint32))
    np.testing.assert_array_equal(conn, ref["conn"])


def test_plans_partition_the_planes():
    for nzn in (2, 3, 7, 30, 1025):
        for world in range(1, min(8, nzn // 2) + 1):
            plans = [SlabPlan(nzn, world, r) for r in range(world)]
            assert plans[0].p0 == 0 and plans[-1].p1 == nzn
            for a, b in zip(plans, plans[1:]):
                assert a.p1 == b.p0 and a.ghost and a.k1 == b.k0 + 1
            assert not plans[-1].ghost
            sizes = [p.p1 - p.p0 for p in plans]
            assert max(sizes) - min(sizes) <= 1
            assert sum(p.nz_cells for p in plans) == nzn - 1
    with pytest.raises(ValueError):
        SlabPlan(3, 2, 0)
    with pytest.raises(ValueError):
        SlabPlan(30, 2, 2)


def test_balanced_bounds():
    """Equal work gives equal runs; a dense band gets short runs; every run
    keeps at least two planes; the bounds partition the planes."""
    assert balanced_bounds(np.ones(1024), 8) == [128 * r for r in range(9)]
    w = np.ones(1024)
    w[400:600] += 50.0
    b = balanced_bounds(w, 8)
    sums = [w[b[i]:b[i + 1]].sum() for i in range(8)]
    assert max(sums) - min(sums) <= 2 * w.max()
    assert b[1] > 300 and b[-2] < 700
    assert balanced_bounds(np.ones(16), 8) == list(range(0, 17, 2))
    spike = np.zeros(40)
    spike[5] = 1e6
    b = balanced_bounds(spike, 4)
    assert b[0] == 0 and b[-1] == 40 and all(b[i + 1] - b[i] >= 2 for i in range(4))
    with pytest.raises(ValueError):
        balanced_bounds(np.ones(7), 4)


def test_rebalanced_bounds():
    """Equal times keep the bounds; a slow rank gives planes to fast ones in
    proportion to its excess over the threshold time per plane; the result
    partitions the same planes with runs of at least two planes."""
    eq = [0, 128, 256, 384, 513]
    assert rebalanced_bounds(eq, [0.08] * 4, [0.16] * 4) == eq
    # Rank 1 takes 10 us more than the others (152.5 us); 0.625 us per plane.
    k1 = [0.080, 0.080, 0.080, 0.0806]
    busy = [0.1525, 0.1625, 0.1525, 0.1525]
    # Mean 155 us: rank 1 sheds 7.5 / 0.625 = 12 planes, the others take 4 each.
    b = rebalanced_bounds(eq, k1, busy, damp=1.0)
    assert b == [0, 132, 248, 380, 513]
    # damp scales the move
    assert rebalanced_bounds(eq, k1, busy, damp=0.5) == [0, 130, 252, 382, 513]
    # a rank that is far too slow still keeps two planes, the runs still partition
    b = rebalanced_bounds([0, 4, 8, 12, 16], [0.004] * 4, [10.0, 0.1, 0.1, 0.1])
    assert b[0] == 0 and b[-1] == 16 and all(b[i + 1] - b[i] >= 2 for i in range(4))
    # bounds not starting at zero keep their ends
    b = rebalanced_bounds([10, 20, 30], [0.01, 0.01], [0.02, 0.03])
    assert b[0] == 10 and b[-1] == 30 and b[1] > 20
    with pytest.raises(ValueError):
        rebalanced_bounds([0, 4, 8], [0.1], [0.1, 0.2])
    with pytest.raises(ValueError):
        rebalanced_bounds([0, 1, 3], [0.1, 0.1], [0.1, 0.1])


@pytest.mark.parametrize("world", [2, 3, 5])
def test_uneven_slabs_assemble_to_single_volume(oracle, world):
    """Slabs on surface-balanced bounds (uneven runs) assemble to the
    single-volume output, like equal runs."""
    vol = _volume()
    isos = [0.0, 1.5, -3.0]
    nzn = SHAPE[2] + 1
    w = np.arange(nzn, dtype=np.float64) ** 2 + 1.0
    bounds = balanced_bounds(w, world)
    plans = [SlabPlan(nzn, world, r, bounds=bounds) for r in range(world)]
    assert [p.p0 for p in plans] + [plans[-1].p1] == bounds
    per = [_rank_counts(oracle, vol, p, isos) for p in plans]
    allc = np.stack([c for c, _, _, _ in per])
    parts = []
    for p, (counts, infos, local, g) in zip(plans, per):
        parts.append(_rank_emit(oracle, local, g, isos, infos, counts, slab_bases(allc, p.rank)))
    _check(parts, _reference(oracle, vol, isos))
    with pytest.raises(ValueError):
        SlabPlan(nzn, world, 0, bounds=bounds[:-1])
    with pytest.raises(ValueError):
        SlabPlan(nzn, 2, 0, bounds=[0, nzn - 1, nzn])


def test_slab_bases_known_answer():
    c = np.array([[[3, 4, 5, 6], [1, 0, 2, 7]],
                  [[10, 20, 30, 40], [0, 1, 0, 2]]], np.int64)   # [world=2, niso=2, 4]
    b = slab_bases(c, 1)
    # isovalue 0: X=13, Y=24, Z=35 -> 72 points; isovalue 1 starts at 72.
    np.testing.assert_array_equal(b["id_base"], [[3, 13 + 4, 13 + 24 + 5],
                                                 [72 + 1, 72 + 1 + 0, 72 + 1 + 1 + 2]])
    np.testing.assert_array_equal(b["out_base"], [[0, 10, 30], [60, 60, 61]])
    np.testing.assert_array_equal(b["tri_out"], [0, 40])
    np.testing.assert_array_equal(b["tri_global"], [6, 46 + 7])
    np.testing.assert_array_equal(b["totals"], [[72, 46], [4, 9]])


@pytest.mark.parametrize("world", [1, 2, 3, 5, 15])
def test_slabs_assemble_to_single_volume(oracle, world):
    """All ranks emulated in one process (gather = stacking the counts)."""
    vol = _volume()
    isos = [0.0, 1.5, -3.0]
    nzn = SHAPE[2] + 1
    plans = [SlabPlan(nzn, world, r) for r in range(world)]
    per = [_rank_counts(oracle, vol, p, isos) for p in plans]
    allc = np.stack([c for c, _, _, _ in per])
    parts = []
    for p, (counts, infos, local, g) in zip(plans, per):
        parts.append(_rank_emit(oracle, local, g, isos, infos, counts, slab_bases(allc, p.rank)))
    _check(parts, _reference(oracle, vol, isos))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, isos, outq):
    import torch.distributed as dist
    from oracle import oracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60))
    try:
        vol = _volume()
        plan = SlabPlan(SHAPE[2] + 1, world, rank)
        counts, infos, local, g = _rank_counts(oracle, vol, plan, isos)
        allc = gather_counts(counts, world)          # the one collective
        part = _rank_emit(oracle, local, g, isos, infos, counts, slab_bases(allc, rank))
        parts = [None] * world
        dist.all_gather_object(parts, part)
        if rank == 0:
            outq.put(parts)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks(oracle):
    """The totals exchange over a real process group (gloo, 2 ranks)."""
    import torch.multiprocessing as mp
    isos = [0.0, 2.0]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    env_path = os.pathsep.join([os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                os.path.dirname(os.path.abspath(__file__))])
    old = os.environ.get("PYTHONPATH")
    os.environ["PYTHONPATH"] = env_path + (os.pathsep + old if old else "")
    try:
        procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, isos, q)) for r in range(2)]
        for p in procs:
            p.start()
        parts = q.get(timeout=120)
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:
        if old is None:
            os.environ.pop("PYTHONPATH", None)
        else:
            os.environ["PYTHONPATH"] = old
    _check(parts, _reference(oracle, _volume(), isos))
