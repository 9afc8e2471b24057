"""Z-slab sharded flying edges: one process per GPU on one node.

The volume is split into contiguous runs of node planes.  Rank r owns node
planes [p0, p1) and also holds plane p1 as a read-only ghost (except the last
rank), so it can close its last layer of cells.  Each rank classifies,
counts and scans its slab independently (tkmc_fe_count with ghost_plane=1);
the only exchange is one gather of 4 int64 totals per isovalue per rank.  By
default (exchange="p2p") that is one small kernel that stores this rank's
totals straight into every other rank's memory over NVLink (CUDA IPC
mappings, epoch flags, bounded wait) and plans in the same launch; with
exchange="nccl" it is an NCCL all-gather followed by a plan kernel.  The
host-side run() uses an all-gather through the process group.  From the
gathered totals every rank computes the global point-id bases of its x, y
and z sections, then emits its points and
triangles into rank-local buffers holding exactly its slices of the global
output.  Point ids in conn are global, and the assembled output is
byte-identical to a single-volume flying_edges call: seams are merged, not
duplicated (unlike flying_edges_multiblock, flying_edges.py:766-832, whose
blocks mesh independently).

Ghost-plane x/y edges belong to the next rank.  This rank's scan also covers
the ghost rows, after its own rows, so their offsets continue from this
rank's own totals -- which is exactly where the next rank's sections start.
"""

import ctypes

import numpy as np
import torch

from . import _lib
from .field import CUDABuffer, Field, f32, i32
from .runtime import current_device, current_stream


class SlabPlan:
    """Node-plane ownership of `rank` among `world` for nz_nodes planes:
    equal runs, or the runs [bounds[r], bounds[r + 1]) when `bounds` (world + 1
    increasing plane indices from 0 to nz_nodes) is given."""

    def __init__(self, nz_nodes, world, rank, bounds=None):
        if not (0 <= rank < world) or nz_nodes < 2 * world:
            raise ValueError(f"cannot split {nz_nodes} planes over {world} ranks")
        self.rank, self.world, self.nz_nodes = rank, world, nz_nodes
        if bounds is None:
            base, rem = divmod(nz_nodes, world)
            self.p0 = rank * base + min(rank, rem)
            self.p1 = self.p0 + base + (1 if rank < rem else 0)
        else:
            b = [int(x) for x in bounds]
            if (len(b) != world + 1 or b[0] != 0 or b[-1] != nz_nodes or
                    any(b[i + 1] - b[i] < 1 for i in range(world)) or b[-1] - b[-2] < 2):
                raise ValueError(f"bad slab bounds {b} for {nz_nodes} planes, {world} ranks")
            self.p0, self.p1 = b[rank], b[rank + 1]
        self.ghost = self.p1 < nz_nodes
        self.k0 = self.p0                      # first local plane
        self.k1 = min(self.p1 + 1, nz_nodes)   # one past the last local plane
        self.nz_cells = self.k1 - self.k0 - 1  # cell layers in the local grid

    @property
    def local_planes(self):
        return self.k1 - self.k0

    def __repr__(self):
        return (f"SlabPlan(rank={self.rank}/{self.world}, own=[{self.p0},{self.p1}), "
                f"local=[{self.k0},{self.k1}), ghost={self.ghost})")


def balanced_bounds(work, world, min_planes=2):
    """Slab bounds for SlabPlan: `world` contiguous runs of node planes whose
    sums of per-plane `work` are as equal as the plane granularity allows
    (each run at least `min_planes` planes).  A plane's work is whatever
    predicts its device time, e.g. a cost per node plus a cost per triangle
    of the cell layer above it (from an earlier count of the same or a
    previous volume)."""
    w = np.asarray(work, np.float64)
    n = w.size
    if world < 1 or n < min_planes * world:
        raise ValueError(f"cannot split {n} planes over {world} ranks")
    c = np.concatenate([[0.0], np.cumsum(w)])
    bounds = [0]
    for r in range(1, world):
        target = c[-1] * r / world
        k = int(np.searchsorted(c, target))
        if k > 0 and (k > n or abs(c[k - 1] - target) <= abs(c[k] - target)):
            k -= 1
        k = min(max(k, bounds[-1] + min_planes), n - (world - r) * min_planes)
        bounds.append(k)
    bounds.append(n)
    return bounds


def rebalanced_bounds(bounds, threshold_ms, busy_ms, damp=0.7, min_planes=2):
    """Slab bounds moved toward equal device time per rank, from what each
    rank measured on the current bounds: busy_ms[r] is rank r's device time
    per step without the wait for the other ranks (threshold + count + emit),
    threshold_ms[r] the part of it that scales with its node planes (the
    threshold read).  A rank above the mean gives up planes, one below takes
    them: (mean - busy) / (threshold time per plane) planes, times `damp`
    (moving planes also moves surface, whose count and emit time the
    threshold slope leaves out, so the full step would overshoot).  Returns
    world + 1 increasing plane indices from 0 to the same last plane; every
    run keeps at least `min_planes` planes.  Meant to be applied once or
    twice; equal times return the same bounds."""
    b = np.asarray(bounds, np.int64)
    n = np.diff(b).astype(np.float64)
    world = n.size
    t = np.asarray(busy_ms, np.float64)
    k1 = np.asarray(threshold_ms, np.float64)
    if world < 1 or t.size != world or k1.size != world or np.any(n < 1):
        raise ValueError(f"bad bounds {list(b)} or times for {world} ranks")
    total = int(b[-1] - b[0])
    if total < min_planes * world:
        raise ValueError(f"cannot split {total} planes over {world} ranks")
    per_plane = float(np.median(k1 / n))
    if not np.isfinite(per_plane) or per_plane <= 0.0:
        return [int(x) for x in b]
    want = n + damp * (t.mean() - t) / per_plane
    want = np.maximum(want, float(min_planes))
    want *= total / want.sum()
    c = np.concatenate([[0.0], np.cumsum(want)])
    out = [int(b[0])]
    for r in range(1, world):
        k = int(b[0]) + int(round(c[r]))
        k = min(max(k, out[-1] + min_planes), int(b[-1]) - (world - r) * min_planes)
        out.append(k)
    out.append(int(b[-1]))
    return out


def slab_bases(all_counts, rank):
    """Offsets of `rank`'s output within the global layout.

    all_counts: int64 [world, niso, 4] = per rank and isovalue {X, Y, Z, T}.
    Global layout is isovalue-major; within an isovalue the x section of
    every rank (in rank order), then all y, then all z -- the single-volume
    layout.  Returns dict of int64 arrays:
      id_base  [niso, 3]  global id of this rank's first x / y / z point
      out_base [niso, 3]  rank-local row of this rank's first x / y / z point
      tri_out  [niso]     rank-local row of this rank's first triangle
      tri_global [niso]   global row of this rank's first triangle
      pt_global_out [niso, 3] global row of the first x/y/z point (== id_base)
      totals   [niso, 2]  global points and triangles per isovalue
    """
    c = np.asarray(all_counts, np.int64)
    world, niso, _ = c.shape
    tot = c.sum(axis=0)                      # [niso, 4]
    P = tot[:, :3].sum(axis=1)               # global points per isovalue
    Pq = np.concatenate([[0], np.cumsum(P)[:-1]])
    Tq = np.concatenate([[0], np.cumsum(tot[:, 3])[:-1]])
    before = c[:rank].sum(axis=0)            # [niso, 4] earlier ranks
    id_base = np.stack([Pq + before[:, 0],
                        Pq + tot[:, 0] + before[:, 1],
                        Pq + tot[:, 0] + tot[:, 1] + before[:, 2]], axis=1)
    own = c[rank]
    own_p = own[:, :3].sum(axis=1)
    lp = np.concatenate([[0], np.cumsum(own_p)[:-1]])
    out_base = np.stack([lp, lp + own[:, 0], lp + own[:, 0] + own[:, 1]], axis=1)
    tri_out = np.concatenate([[0], np.cumsum(own[:, 3])[:-1]])
    return {"id_base": id_base, "out_base": out_base, "tri_out": tri_out,
            "tri_global": Tq + before[:, 3], "pt_global_out": id_base,
            "totals": np.stack([P, tot[:, 3]], axis=1)}


def gather_counts(counts, world, group=None, device=None, out=None):
    """All-gather every rank's totals: ONE collective of 4 int64 per
    isovalue per rank.  counts: int64 [niso, 4] on the host.  device is the
    process group's device (a CUDA device for NCCL, cpu for gloo); out an
    optional preallocated [world*niso*4] int64 tensor there.  Returns int64
    [world, niso, 4] on the host."""
    import torch.distributed as dist
    c = np.ascontiguousarray(np.asarray(counts, np.int64).reshape(-1))
    niso = c.size // 4
    if world == 1:
        return c.reshape(1, niso, 4)
    device = torch.device("cpu") if device is None else device
    src = torch.from_numpy(c).to(device)
    if out is None:
        out = torch.empty(world * c.size, dtype=torch.int64, device=device)
    dist.all_gather_into_tensor(out, src, group=group)
    return out.cpu().numpy().reshape(world, niso, 4)


def _i64(vals):
    flat = [int(v) for v in np.asarray(vals).reshape(-1)]
    return (ctypes.c_int64 * len(flat))(*flat)


def _f32(vals):
    return (ctypes.c_float * len(vals))(*[float(v) for v in vals])


class SlabEngine:
    """Per-rank state: plan, workspace and the collective used for totals."""

    def __init__(self, grid, plan, isovalues, group=None, exchange="nccl"):
        """exchange: how run_device shares the totals between ranks --
        "nccl" (an all-gather into device buffers) or "p2p" (one kernel
        storing into every rank's memory over NVLink; needs one GPU per rank
        and CUDA IPC between the processes)."""
        if len(isovalues) > _lib.MAX_ISO:
            raise ValueError(f"at most {_lib.MAX_ISO} isovalues per slab call")
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"unknown exchange {exchange!r}")
        self.grid, self.plan, self.isos = grid, plan, list(isovalues)
        self.group = group
        self.exchange_kind = exchange
        self._xchg = None
        self.dev = current_device()
        self.lib = _lib.load()
        nx, ny = grid.nx, grid.ny
        self.nbytes = self.lib.tkmc_fe_workspace_bytes(nx, ny, plan.nz_cells, len(self.isos))
        self.ws = torch.empty(self.nbytes, dtype=torch.uint8, device=self.dev)
        world = plan.world
        self.gathered = torch.zeros(world * len(self.isos) * 4, dtype=torch.int64,
                                    device=self.dev)
        # Device-side plan: this rank's totals and its output bases.
        self.counts_dev = torch.zeros(len(self.isos) * 4, dtype=torch.int64, device=self.dev)
        self.bases_dev = torch.zeros(len(self.isos) * 7, dtype=torch.int64, device=self.dev)
        self._xstream = None
        if exchange == "p2p" and world > 1:
            self._xstream = torch.cuda.Stream(self.dev)
            self._connect_p2p()

    def _connect_p2p(self):
        """Create this rank's exchange buffer and open every rank's (their
        IPC handles travel once through the process group)."""
        import torch.distributed as dist
        p, lib = self.plan, self.lib
        x = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(lib.tkmc_exchange_handle_bytes())
        _lib.check(lib.tkmc_exchange_create(p.world, p.rank, len(self.isos), ctypes.byref(x),
                                            handle), "tkmc_exchange_create")
        self._xchg = x
        handles = [None] * p.world
        dist.all_gather_object(handles, handle.raw, group=self.group)
        allh = ctypes.create_string_buffer(b"".join(handles))
        _lib.check(lib.tkmc_exchange_connect(x, allh), "tkmc_exchange_connect")

    def close(self):
        """Release the exchange buffer.  Every rank calls it after its last
        run_device (it synchronises with the other ranks first)."""
        if self._xchg is not None:
            import torch.distributed as dist
            torch.cuda.synchronize(self.dev)
            dist.barrier(group=self.group)
            self.lib.tkmc_exchange_destroy(self._xchg)
            self._xchg = None

    def count(self, local_values):
        g, p, lib = self.grid, self.plan, self.lib
        niso = len(self.isos)
        counts = np.zeros(niso * 4, np.int64)
        _lib.check(lib.tkmc_fe_count(local_values.data_ptr(), g.nx, g.ny, p.nz_cells,
                                     1 if p.ghost else 0, _f32(self.isos), niso, None,
                                     self.ws.data_ptr(), self.nbytes, counts.ctypes.data,
                                     current_stream(self.dev)), "tkmc_fe_count")
        return counts.reshape(niso, 4)

    def plane_triangles(self, counts):
        """Triangles of the cell layer above each own node plane (all
        isovalues), from the last count on this engine; counts is that
        count's [niso, 4] totals.  Copies the row table to the host
        (synchronises)."""
        g, p, lib = self.grid, self.plan, self.lib
        niso = len(self.isos)
        rows = (g.ny + 1) * (p.nz_cells + 1)
        own = p.p1 - p.p0
        out = np.zeros(rows * 4, np.int64)
        tris = np.zeros(own, np.int64)
        for q in range(niso):
            _lib.check(lib.tkmc_fe_row_offsets(g.nx, g.ny, p.nz_cells, niso, q, self.ws.data_ptr(),
                                               self.nbytes, out.ctypes.data,
                                               current_stream(self.dev)), "tkmc_fe_row_offsets")
            per_row = np.diff(np.append(out.reshape(rows, 4)[:, 3], int(counts[q, 3])))
            tris += per_row.reshape(p.nz_cells + 1, g.ny + 1)[:own].sum(axis=1)
        return tris

    def exchange(self, counts):
        """All-gather every rank's totals (one collective)."""
        return gather_counts(counts, self.plan.world, self.group, self.dev, self.gathered)

    def emit(self, local_values, counts, bases):
        g, p, lib = self.grid, self.plan, self.lib
        own_p = int(counts[:, :3].sum())
        own_t = int(counts[:, 3].sum())
        pts = torch.empty(max(own_p, 1) * 3, dtype=torch.float32, device=self.dev)
        conn = torch.empty(max(own_t, 1) * 3, dtype=torch.int32, device=self.dev)
        if own_p or own_t:
            _lib.check(lib.tkmc_fe_emit(
                local_values.data_ptr(), g.nx, g.ny, p.nz_cells, 1 if p.ghost else 0, p.k0,
                _f32([g.x0, g.y0, g.z0, g.dx, g.dy, g.dz]), _f32(self.isos), len(self.isos),
                None, self.ws.data_ptr(), self.nbytes, _i64(bases["id_base"]),
                _i64(bases["out_base"]), _i64(bases["tri_out"]), pts.data_ptr(), own_p,
                conn.data_ptr(), own_t, current_stream(self.dev)), "tkmc_fe_emit")
        return pts[:own_p * 3], conn[:own_t * 3]

    def run_device(self, local_values, points, conn, counts_host=None, marks=None):
        """classify -> count -> totals exchange and plan -> emit, with nothing
        read on the host in between.  With the peer exchange the count pass
        is split: the exchange kernel runs on a second stream right after
        the per-row counts, while the offsets pass runs on this one, and the
        emit waits for both.  Otherwise: the offsets pass, the totals copied
        to a device array (with several ranks, NCCL-all-gathered), a plan
        kernel.  points / conn
        are flat f32 / int32 CUDA tensors whose sizes are the capacities;
        writes past them are skipped and reported by check().  When
        counts_host (pinned int64, niso*4) is given, this rank's totals are
        copied there asynchronously.  Every rank takes the same collective
        (or peer exchange) each call.
        marks: optional 5 CUDA events, recorded before the classify, the
        count, after the offsets pass, when the bases are ready (the wait
        for the exchange) and after the emit (phase timing)."""
        import torch.distributed as dist
        g, p, lib = self.grid, self.plan, self.lib
        niso = len(self.isos)
        st = current_stream(self.dev)
        isos = _f32(self.isos)
        ghost = 1 if p.ghost else 0

        def mark(i):
            if marks is not None:
                marks[i].record(torch.cuda.current_stream(self.dev))

        mark(0)
        _lib.check(lib.tkmc_fe_classify(local_values.data_ptr(), g.nx, g.ny, p.nz_cells, isos,
                                        niso, self.ws.data_ptr(), self.nbytes, st),
                   "tkmc_fe_classify")
        mark(1)
        bases = self.bases_dev.data_ptr()
        if self._xchg is not None:
            # Totals over NVLink peer stores, plan in the same kernel, on a
            # second stream as soon as the count pass is done: the exchange
            # (and the wait for the slowest rank) overlaps the offsets pass.
            _lib.check(lib.tkmc_fe_scan_part(g.nx, g.ny, p.nz_cells, ghost, niso, None,
                                             self.ws.data_ptr(), self.nbytes, 1, st),
                       "tkmc_fe_scan_part")
            main = torch.cuda.current_stream(self.dev)
            self._xstream.wait_stream(main)
            _lib.check(lib.tkmc_exchange_plan_counts(self._xchg, g.nx, g.ny, p.nz_cells, ghost,
                                                     self.ws.data_ptr(), self.nbytes, 0, bases,
                                                     self._xstream.cuda_stream),
                       "tkmc_exchange_plan_counts")
            _lib.check(lib.tkmc_fe_scan_part(g.nx, g.ny, p.nz_cells, ghost, niso, None,
                                             self.ws.data_ptr(), self.nbytes, 2, st),
                       "tkmc_fe_scan_part")
            mark(2)
            main.wait_stream(self._xstream)
        else:
            _lib.check(lib.tkmc_fe_scan(g.nx, g.ny, p.nz_cells, ghost, niso, None,
                                        self.ws.data_ptr(), self.nbytes, st), "tkmc_fe_scan")
            mark(2)
        if self._xchg is None:
            _lib.check(lib.tkmc_fe_copy_counts(g.nx, g.ny, p.nz_cells, niso, self.ws.data_ptr(),
                                               self.nbytes, self.counts_dev.data_ptr(), st),
                       "tkmc_fe_copy_counts")
            src = self.counts_dev
            if p.world > 1:
                dist.all_gather_into_tensor(self.gathered, self.counts_dev, group=self.group)
                src = self.gathered
            _lib.check(lib.tkmc_fe_plan(src.data_ptr(), p.world, p.rank, niso, 0, bases, st),
                       "tkmc_fe_plan")
        mark(3)
        _lib.check(lib.tkmc_fe_emit_dev(
            local_values.data_ptr(), g.nx, g.ny, p.nz_cells, ghost, p.k0,
            _f32([g.x0, g.y0, g.z0, g.dx, g.dy, g.dz]), isos, niso, None, self.ws.data_ptr(),
            self.nbytes, bases, points.data_ptr(), points.numel() // 3,
            conn.data_ptr(), conn.numel() // 3, st), "tkmc_fe_emit_dev")
        mark(4)
        if counts_host is not None:
            _lib.check(lib.tkmc_fe_copy_counts(g.nx, g.ny, p.nz_cells, niso, self.ws.data_ptr(),
                                               self.nbytes, counts_host.data_ptr(), st),
                       "tkmc_fe_copy_counts")

    def capture(self, local_values, points, conn, counts_host=None):
        """Record run_device into a CUDA graph; each replay() is one isosurface
        of local_values (same buffers) with a single launch from the host.
        With several ranks the graph holds the totals all-gather: every rank
        captures together and replays the same number of times, and the
        graph is released before the process group is destroyed."""
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            self.run_device(local_values, points, conn, counts_host)
        torch.cuda.current_stream(self.dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.run_device(local_values, points, conn, counts_host)
        return graph

    def check(self):
        """Synchronise and raise if the device recorded an error."""
        g, p = self.grid, self.plan
        _lib.check(self.lib.tkmc_fe_check(g.nx, g.ny, p.nz_cells, len(self.isos),
                                          self.ws.data_ptr(), self.nbytes,
                                          current_stream(self.dev)), "tkmc_fe_check")

    def run(self, local_values, check=True):
        """count -> all-gather totals -> emit.  Returns this rank's slices."""
        counts = self.count(local_values)
        allc = self.exchange(counts)
        if allc.max() > np.iinfo(np.int32).max or \
                int(allc[:, :, :3].sum()) > np.iinfo(np.int32).max:
            raise OverflowError("global point total does not fit int32 point ids")
        b = slab_bases(allc, self.plan.rank)
        pts, conn = self.emit(local_values, counts, b)
        if check:
            self.check()
        return {"points_field": Field(f32, (pts.numel(),), CUDABuffer(pts)),
                "conn_field": Field(i32, (conn.numel(),), CUDABuffer(conn)),
                "counts": counts, "all_counts": allc, "bases": b,
                "total_points": int(b["totals"][:, 0].sum()),
                "total_tris": int(b["totals"][:, 1].sum())}


def flying_edges_zslab(local_values, grid, plan, isovalues, group=None):
    """Sharded isosurface of one rank's slab; see module docstring.

    local_values: f32 CUDA tensor of planes [plan.k0, plan.k1) of the whole
    volume (grid = the whole volume's UniformGrid).
    """
    return SlabEngine(grid, plan, isovalues, group).run(local_values)


def assemble(parts):
    """Host-side assembly of every rank's result into the single-volume
    output (points (P,3), conn (T,3)).  parts: per rank a dict with numpy
    'points' (flat), 'conn' (flat), 'counts' [niso,4] and 'bases'."""
    b0 = parts[0]["bases"]
    P = int(b0["totals"][:, 0].sum())
    T = int(b0["totals"][:, 1].sum())
    points = np.empty((P, 3), np.float32)
    conn = np.empty((T, 3), np.int32)
    for part in parts:
        c, b = part["counts"], part["bases"]
        pts = np.asarray(part["points"]).reshape(-1, 3)
        cn = np.asarray(part["conn"]).reshape(-1, 3)
        for q in range(c.shape[0]):
            for s in range(3):
                n = int(c[q, s])
                lo = int(b["out_base"][q, s])
                go = int(b["pt_global_out"][q, s])
                points[go:go + n] = pts[lo:lo + n]
            n = int(c[q, 3])
            lo = int(b["tri_out"][q])
            go = int(b["tri_global"][q])
            conn[go:go + n] = cn[lo:lo + n]
    return points, conn
