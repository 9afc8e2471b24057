"""One rank of the z-slab flying-edges path under torchrun (NCCL).

Each rank generates only its own planes (plus the ghost plane) of a 256^3
blobs volume, runs SlabEngine (count -> one all-gather of totals -> emit)
and sends its slices to rank 0, which assembles them and compares the result
with a single-volume flying_edges call on its own GPU.  Each rank also
replays the device-planned step from a CUDA graph (the NCCL all-gather of the
totals inside it), then runs it with the totals exchanged over NVLink peer
stores (once directly, three times from a graph, then four steps alternating
between two different volumes), and checks that every run writes that
volume's slices.  Rank 0 writes "ok" to the file named by argv[1] when they
are identical.
"""

import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import tack_b200 as tack  # noqa: E402
from tack_b200 import workloads  # noqa: E402
from tack_b200.distributed import SlabEngine, SlabPlan, assemble  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    ok = False
    try:
        tack.init(tack.cuda)
        shape = (256, 256, 256)
        nx, ny, nz = shape[0] - 1, shape[1] - 1, shape[2] - 1
        grid = tack.UniformGrid(nx, ny, nz, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
        plan = SlabPlan(shape[2], world, rank)
        vals = workloads.generate("blobs", shape, plan.k0, plan.k1)
        eng = SlabEngine(grid, plan, [0.5])
        r = eng.run(vals)
        part = {"points": r["points_field"].tensor.cpu().numpy(),
                "conn": r["conn_field"].tensor.cpu().numpy(),
                "counts": r["counts"], "bases": r["bases"]}
        # The device-planned step captured in a CUDA graph, NCCL all-gather
        # inside, replayed twice: the same slices.
        pts = torch.zeros_like(r["points_field"].tensor)
        conn = torch.zeros_like(r["conn_field"].tensor)
        graph = eng.capture(vals, pts, conn)
        for _ in range(2):
            pts.zero_()
            graph.replay()
        torch.cuda.synchronize()
        eng.check()
        graph_ok = (torch.equal(pts.view(torch.int32), r["points_field"].tensor.view(torch.int32))
                    and torch.equal(conn, r["conn_field"].tensor))
        del graph
        # The same step with the totals exchanged over NVLink peer stores.
        eng2 = SlabEngine(grid, plan, [0.5], exchange="p2p")
        pts.zero_()
        eng2.run_device(vals, pts, conn)
        torch.cuda.synchronize()
        eng2.check()
        graph_ok = graph_ok and torch.equal(pts.view(torch.int32),
                                            r["points_field"].tensor.view(torch.int32))
        graph = eng2.capture(vals, pts, conn)
        for _ in range(3):
            pts.zero_()
            graph.replay()
        torch.cuda.synchronize()
        eng2.check()
        graph_ok = graph_ok and torch.equal(pts.view(torch.int32),
                                            r["points_field"].tensor.view(torch.int32)) and \
            torch.equal(conn, r["conn_field"].tensor)
        del graph
        # Steps over two different volumes in turn: every exchange carries
        # new totals, and each step's slices must match that volume's
        # host-planned run.
        vals_b = (vals * 1.25).contiguous()
        rb = eng.run(vals_b)
        pts_b = torch.zeros_like(rb["points_field"].tensor)
        conn_b = torch.zeros_like(rb["conn_field"].tensor)
        for i in range(4):
            src, p_out, c_out, ref_r = ((vals, pts, conn, r) if i % 2 == 0
                                        else (vals_b, pts_b, conn_b, rb))
            p_out.zero_()
            eng2.run_device(src, p_out, c_out)
            torch.cuda.synchronize()
            eng2.check()
            graph_ok = graph_ok and torch.equal(
                p_out.view(torch.int32), ref_r["points_field"].tensor.view(torch.int32)) and \
                torch.equal(c_out, ref_r["conn_field"].tensor)
        eng2.close()
        flags = [None] * world
        dist.all_gather_object(flags, graph_ok)
        parts = [None] * world
        dist.all_gather_object(parts, part)
        if rank == 0:
            points, conn = assemble(parts)
            whole = workloads.generate("blobs", shape)
            ref = tack.flying_edges(tack.from_torch(whole), grid, 0.5)
            ok = (np.array_equal(conn, ref["conn"]) and
                  np.array_equal(points.view(np.uint32), ref["points"].view(np.uint32)) and
                  all(flags))
            with open(sys.argv[1], "w") as f:
                f.write("ok\n" if ok else "mismatch\n")
        dist.barrier()
    finally:
        dist.destroy_process_group()
    return 0 if (ok or rank != 0) else 1


if __name__ == "__main__":
    sys.exit(main())
