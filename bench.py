#!/usr/bin/env python
"""Isosurface throughput on B200: input Gcells/s of flying-edges marching cubes.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tack_b200|reference]

Workload (default): 1024^3 f32 volume, sum of 32 seeded Gaussian blobs,
isovalue 0.5 -- the configuration the metric is quoted on at 1/2/4/8 GPUs.
The volume is z-slab sharded across N GPUs (one process per GPU, launched by
torchrun for N > 1): each rank classifies/counts/scans its slab, one NCCL
all-gather exchanges the per-rank totals, each rank emits its slices of the
single-volume output.  Total work is fixed as N grows (strong scaling).

A step = one isosurface of the whole volume from resident f32 values to
resident points + connectivity: classify, count + scan, the per-rank totals
all-gathered on the device, device-side planning of the output bases, emit,
and an asynchronous copy of the totals to pinned host memory.  Output buffers
are allocated once, at this volume's exact size, from one host-planned run
before the timed steps (as when a caller processes a sequence of volumes);
every step's totals are checked against it afterwards.  `value` = cells of
the whole volume per second over K timed steps (CUDA events, max over ranks).  `e2e` = the same metric
through the public API from pinned host memory: each step copies the volume
host->device, runs flying_edges, copies points and connectivity back.

The reference arm (--impl reference) times the CPU parity oracle -- a C
restatement of the reference's flying-edges kernels with its host
orchestration, using every host core -- on a bounded z-slab of the same
volume (the reference itself is a Python package whose JIT path cannot be
shipped to the GPU host).
"""

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

METRIC = "isosurface input Gcells/s at 1/2/4/8 B200; achieved HBM GB/s vs peak"
TRAFFIC_FILE = os.path.join(REPO, "profiles", "fe_threshold_blobs1024.txt")
# Relative device time per node (threshold read, 4 B at ~6.5 TB/s: 0.6 ps) and
# per triangle (count + emit: 0.27 ms for 5.3 M triangles, 51 ps) on one
# B200 at 1024^3 blobs; used to balance z-slabs at N > 1.
NODE_COST, TRI_COST = 1.0, 83.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="tack_b200", choices=["tack_b200", "reference"])
    ap.add_argument("--config", default="blobs")
    ap.add_argument("--size", type=int, nargs=3, default=None,
                    help="override the volume's node counts (nx ny nz)")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="totals exchange between ranks (N>1): NVLink peer stores or NCCL")
    ap.add_argument("--balance-slabs", action="store_true",
                    help="N>1: node-plane runs balanced by the surface of a first pass "
                         "instead of equal runs")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, STREAM-style copy)"
    return 6650.0, "fallback (6.65 TB/s, earlier measurement on this pool)"


def committed_traffic():
    """DRAM bytes per launch of the threshold kernel from the committed ncu
    summary (a line 'dram_bytes_per_launch_1024cubed: N'), or None."""
    if not os.path.exists(TRAFFIC_FILE):
        return None
    for line in open(TRAFFIC_FILE):
        if line.startswith("dram_bytes_per_launch_1024cubed:"):
            return float(line.split(":", 1)[1].split()[0])
    return None


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """SM clock, power and clock-event reasons of this rank's GPU, read through
    NVML (reads only) by a thread every ~2 ms while the timed steps run, plus
    one sample taken by the caller while queued steps are still executing
    (``sample_now``), so a short timed region still has a sample under load.
    Falls back to ``nvidia-smi -lms`` when NVML cannot be opened."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.nvml = self.handle = None
        self.rows = []          # (sm_mhz, max_mhz, power_w, reason bits)
        self.thread = self.halt = None
        self.proc = self.path = None

    def _open_nvml(self):
        import torch
        import pynvml
        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(self.dev)
        bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        self.nvml = pynvml

    def sample_now(self):
        if self.nvml is None:
            return
        n, h = self.nvml, self.handle
        try:
            get_reasons = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                n.nvmlDeviceGetCurrentClocksThrottleReasons
            self.rows.append((n.nvmlDeviceGetClockInfo(h, n.NVML_CLOCK_SM),
                              n.nvmlDeviceGetMaxClockInfo(h, n.NVML_CLOCK_SM),
                              n.nvmlDeviceGetPowerUsage(h) / 1000.0, int(get_reasons(h))))
        except Exception:
            pass

    def start(self):
        import threading
        try:
            self._open_nvml()
        except Exception:
            self.nvml = None
        if self.nvml is not None:
            self.halt = threading.Event()

            def loop():
                while not self.halt.is_set():
                    self.sample_now()
                    self.halt.wait(0.002)
            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return
        import tempfile
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.dev)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.halt.set()
            self.thread.join(timeout=5)
            rows = self.rows
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
            if not rows:
                return {"samples": 0, "source": "nvml"}
            return {"sm_mhz": statistics.median(r[0] for r in rows),
                    "sm_max_mhz": max(r[1] for r in rows),
                    "power_w": round(statistics.median(r[2] for r in rows), 1),
                    "reasons": sorted({nm for r in rows for nm, bit in self.REASONS if r[3] & bit}),
                    "samples": len(rows), "source": "nvml"}
        if self.proc is None:
            return {"samples": 0, "note": "neither NVML nor nvidia-smi available"}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"samples": 0, "source": "nvidia-smi"}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = [nm for nm, _ in self.REASONS]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "source": "nvidia-smi"}


# ---------------------------------------------------------------- reference arm

def cpu_sample_rate(volume_host_planes, shape, k0, isos, nthreads, min_seconds, max_calls=50):
    """Oracle flying_edges on a z-slab; returns (Gcells/s, per-call seconds, cells)."""
    from oracle import oracle
    nx, ny, _ = shape
    nz_cells = volume_host_planes.size // (nx * ny) - 1
    g = oracle.Grid(nx - 1, ny - 1, nz_cells, 0.0, 0.0, float(k0), 1.0, 1.0, 1.0)
    cells = (nx - 1) * (ny - 1) * nz_cells
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        oracle.flying_edges_isovalues(volume_host_planes, g, isos, nthreads=nthreads)
        times.append(time.perf_counter() - t0)
        if (time.perf_counter() - t_start >= min_seconds and len(times) >= 3) or \
                len(times) >= max_calls:
            break
    t = statistics.median(times)
    return cells / t / 1e9, t, cells


def host_slab(args, shape, planes, device):
    """The middle `planes` node planes of the workload, as a host array."""
    from tack_b200 import workloads
    nz = shape[2]
    k0 = max(0, nz // 2 - planes // 2)
    v = workloads.generate(args.config, shape, k0, k0 + planes, device=device)
    return v.cpu().numpy(), k0


def run_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    import torch
    from oracle import oracle
    from tack_b200 import workloads
    oracle.build()
    cfg = workloads.CONFIGS[args.config]
    shape = tuple(args.size) if args.size else cfg["shape"]
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    nthreads = oracle.num_threads(0)
    # Size the slab so that warmup + steps fit in about two minutes.
    calib, k0 = host_slab(args, shape, 8, device)
    rate, _, _ = cpu_sample_rate(calib, shape, k0, cfg["isovalues"], nthreads, 0.0, max_calls=2)
    budget = 120.0 / max(1, args.steps + args.warmup)
    cells_per_plane = (shape[0] - 1) * (shape[1] - 1)
    planes = int(np.clip(budget * rate * 1e9 / cells_per_plane, 2, min(128, shape[2])))
    vol, k0 = host_slab(args, shape, planes, device)
    nz_cells = planes - 1
    g = oracle.Grid(shape[0] - 1, shape[1] - 1, nz_cells, 0.0, 0.0, float(k0), 1.0, 1.0, 1.0)
    cells = cells_per_plane * nz_cells
    for _ in range(args.warmup):
        oracle.flying_edges_isovalues(vol, g, cfg["isovalues"], nthreads=nthreads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.flying_edges_isovalues(vol, g, cfg["isovalues"], nthreads=nthreads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = cells * args.steps / total / 1e9
    sample = (f"node planes [{k0},{k0 + planes}) of the {shape[0]}x{shape[1]}x{shape[2]} "
              f"{args.config} volume ({cells} cells) per step")
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "Gcells/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args.config, shape, cfg["isovalues"]),
                   "volume_nodes": list(shape), "isovalues": cfg["isovalues"]},
        "cpu_baseline": {"value": value, "unit": "Gcells/s", "cores": nthreads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "Gcells/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": ("CPU parity oracle (C restatement of the reference's flying-edges kernels "
                 "and host orchestration, pthreads over rows), all host threads"),
    }
    print(json.dumps(out), flush=True)
    return 0


def workload_name(config, shape, isos):
    desc = {"blobs": "sum of 32 seeded Gaussian blobs", "gyroid": "gyroid + N(0,0.01) noise",
            "sines": "sum of 8 seeded sinusoids", "sphere": "sphere SDF",
            "noise": "4-octave value noise"}[config]
    return (f"flying-edges isosurface, {shape[0]}x{shape[1]}x{shape[2]} f32 volume, {desc}, "
            f"isovalue(s) {isos}")


# ---------------------------------------------------------------- GPU arm

def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    import torch
    import torch.distributed as dist

    import tack_b200 as tack
    from tack_b200 import _lib, workloads
    from tack_b200.distributed import SlabEngine, SlabPlan, balanced_bounds, slab_bases

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    tack.init(tack.cuda, device=local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    cfg = workloads.CONFIGS[args.config]
    shape = tuple(args.size) if args.size else cfg["shape"]
    isos = cfg["isovalues"]
    nxn, nyn, nzn = shape
    plan = SlabPlan(nzn, world, rank)
    grid = tack.UniformGrid(nxn - 1, nyn - 1, nzn - 1, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
    vol = workloads.generate(args.config, shape, plan.k0, plan.k1, device=dev)
    torch.cuda.synchronize()
    eng = SlabEngine(grid, plan, isos, exchange=args.exchange)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    niso = len(isos)
    isoc = (ctypes_f32(isos))
    local_nodes = vol.numel()
    cells = (nxn - 1) * (nyn - 1) * (nzn - 1)

    # Output buffers of this rank's exact size, from one host-planned run;
    # the timed steps then run count -> plan -> emit with no host round trip
    # (the totals reach the host asynchronously, as a caller would read them).
    first = eng.run(vol)
    own = first["counts"]
    balanced = None
    if world > 1 and args.balance_slabs:
        # Slab bounds balanced by predicted device time: the surface of this
        # first pass (in a time series, the previous step's) gives each node
        # plane's triangles; a plane costs NODE_COST per node (the threshold
        # read) plus TRI_COST per triangle (count and emit).  Then the slabs
        # are set up again on the new bounds.
        tris = eng.plane_triangles(own)
        allt = [None] * world
        dist.all_gather_object(allt, tris.tolist())
        plane_tris = np.concatenate([np.asarray(t, np.float64) for t in allt])
        work = NODE_COST * nxn * nyn + TRI_COST * plane_tris
        balanced = balanced_bounds(work, world)
        eng.close()
        del eng, vol, first
        plan = SlabPlan(nzn, world, rank, bounds=balanced)
        vol = workloads.generate(args.config, shape, plan.k0, plan.k1, device=dev)
        torch.cuda.synchronize()
        eng = SlabEngine(grid, plan, isos, exchange=args.exchange)
        local_nodes = vol.numel()
        first = eng.run(vol)
        own = first["counts"]
    own_p, own_t = int(own[:, :3].sum()), int(own[:, 3].sum())
    pts_buf = torch.empty(max(own_p, 1) * 3, dtype=torch.float32, device=dev)
    conn_buf = torch.empty(max(own_t, 1) * 3, dtype=torch.int32, device=dev)
    counts_host = torch.zeros(niso * 4, dtype=torch.int64, pin_memory=True)
    bases = first["bases"]
    ev = {}

    def step(i=None):
        marks = [ev[k][i] for k in "abcde"] if i is not None else None
        eng.run_device(vol, pts_buf, conn_buf, counts_host, marks)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    K = args.steps
    # Phase times: CUDA events between the phases of ordinary (not graph)
    # steps, after the warm-up; the headline time is measured below.
    KP = min(K, 50)
    for key in "abcde":
        ev[key] = [torch.cuda.Event(enable_timing=True) for _ in range(KP)]
    for i in range(KP):
        step(i)
    torch.cuda.synchronize()
    k1 = sum(ev["a"][i].elapsed_time(ev["b"][i]) for i in range(KP)) / KP
    k2 = sum(ev["b"][i].elapsed_time(ev["c"][i]) for i in range(KP)) / KP
    k3 = sum(ev["d"][i].elapsed_time(ev["e"][i]) for i in range(KP)) / KP
    host = sum(ev["c"][i].elapsed_time(ev["d"][i]) for i in range(KP)) / KP  # totals + plan
    # The whole step, the totals all-gather included, is one CUDA graph: one
    # host launch per step on every rank.
    launches0 = lib.tkmc_launch_count()
    barrier()
    graph = eng.capture(vol, pts_buf, conn_buf, counts_host)
    torch.cuda.synchronize()
    per_step = lib.tkmc_launch_count() - launches0
    per_step //= 2  # capture() runs the step once before recording it

    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    barrier()
    clocks.start()
    launches0 = lib.tkmc_launch_count()
    t_start.record(stream)
    for i in range(K):
        graph.replay()
    t_end.record(stream)
    clocks.sample_now()  # the queued steps are still running
    torch.cuda.synchronize()
    launches = per_step * K
    eng.check()  # any device-recorded error (capacity, timeout) invalidates the run
    if not np.array_equal(counts_host.numpy().reshape(niso, 4), own):
        raise RuntimeError("device-planned steps disagree with the host-planned run")
    clk = clocks.stop()
    barrier()
    ms = t_start.elapsed_time(t_end)
    del graph
    # The threshold kernel's roofline at N > 1: the rank with the lowest
    # achieved bandwidth (slabs can differ in size), with its own bytes.
    k1_rank = torch.tensor([4.0 * local_nodes / (k1 * 1e-3), float(local_nodes), k1],
                           dtype=torch.float64, device=dev)
    if world > 1:
        allk1 = [torch.zeros_like(k1_rank) for _ in range(world)]
        dist.all_gather(allk1, k1_rank)
        k1_rank = min(allk1, key=lambda t: float(t[0]))
    k1_nodes, k1_ms = float(k1_rank[1]), float(k1_rank[2])
    stats = torch.tensor([ms, k1, k2, k3, host], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms, k1, k2, k3, host = (float(x) for x in stats.cpu())
    total_points = int(bases["totals"][:, 0].sum())
    total_tris = int(bases["totals"][:, 1].sum())

    # ---- next filter on the same surface: vertex normals (one GPU) --------
    normals = soup = None
    if world == 1 and own_p > 0 and own_t > 0:
        normals = time_normals(tack, torch, pts_buf[:own_p * 3], conn_buf[:own_t * 3], own_p,
                               own_t, stream)
        soup = time_soup(tack, torch, vol, grid, isos, cells, stream)

    # ---- e2e through the public API, host buffers -------------------------
    e2e = None
    if not args.no_e2e and args.e2e_steps > 0:
        e2e = run_e2e(args, tack, torch, dist, vol, grid, plan, eng, isos, world, rank, dev,
                      cells)

    # ---- CPU baseline (oracle, host cores), N == 1 only ------------------------
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        from oracle import oracle
        oracle.build()
        nthreads = oracle.num_threads(0)
        planes = min(64, nzn)
        k0 = max(0, nzn // 2 - planes // 2)
        slab = vol.view(nzn, nyn, nxn)[k0:k0 + planes].reshape(-1).cpu().numpy()
        rate, t_call, scells = cpu_sample_rate(slab, shape, k0, isos, nthreads, args.cpu_seconds)
        cpu = {"value": rate, "unit": "Gcells/s", "cores": nthreads, "kind": "port",
               "sample": (f"node planes [{k0},{k0 + planes}) of the same volume "
                          f"({scells} cells), median of repeated calls over "
                          f">= {args.cpu_seconds:.0f} s"),
               "seconds_per_call": t_call}

    if world > 1:
        dist.barrier()
    if rank == 0:
        peak, peak_src = measured_peaks()
        alg_k1 = 4.0 * k1_nodes  # one read of that rank's slab (incl. ghost)
        achieved = alg_k1 / (k1_ms * 1e-3) / 1e9
        traffic = committed_traffic()
        if traffic is not None:
            traffic = traffic * k1_nodes / float(1024 ** 3)
        step_bytes = 4.0 * nxn * nyn * nzn + 12.0 * (total_points + total_tris)
        value = cells * K / (ms * 1e-3) / 1e9
        out = {
            "metric": METRIC, "value": value, "unit": "Gcells/s", "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": ms / K,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {
                "workload": workload_name(args.config, shape, isos),
                "volume_nodes": list(shape), "cells": cells, "isovalues": isos,
                "parallelism": (f"z-slab x{world} (ghost plane; totals exchanged by "
                                f"{'NVLink peer stores' if args.exchange == 'p2p' else 'NCCL all-gather'}; "
                                f"{'equal plane runs' if balanced is None else 'plane runs balanced by surface'})"
                                if world > 1 else "single GPU"),
                "slab_bounds": balanced,
                "l2": (f"inputs larger than L2 (f32 slab {4.0 * local_nodes / 2**30:.2f} GiB per "
                       f"GPU vs 126 MB L2), no flush" if 4.0 * local_nodes > 126e6 * 2 else
                       "input smaller than 2x L2: numbers include L2 reuse between steps"),
            },
            "roofline": {
                "bound": "hbm", "kernel": "k_fe_threshold_words (K1: volume -> node bitmask)",
                "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": traffic, "peak_source": peak_src,
                "algorithmic_bytes_per_launch": alg_k1,
                "launch_ms": k1_ms,
            },
            "step_roofline": {
                "algorithmic_bytes": step_bytes,
                "achieved_gbs": step_bytes / (ms / K * 1e-3) / 1e9,
                "frac_of_aggregate_peak": step_bytes / (ms / K * 1e-3) / 1e9 / (peak * world),
            },
            "kernels_ms": {"k1_threshold": k1, "k2_count_scan": k2,
                           "totals_gather_plan": host, "k3_emit": k3},
            "outputs": {"points": total_points, "triangles": total_tris},
            "compute_normals": normals,
            "marching_cubes_soup": soup,
            "gpu_launches": int(launches),
            "gpu_launches_per_step": launches / K,
            "cuda_graph": True,
            "clocks": clk,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(out), flush=True)
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def time_normals(tack, torch, points, conn, n_pts, n_tris, stream, reps=20):
    """tack_b200.compute_normals on the bench's surface: device time per call
    (CUDA events) and its algorithmic bytes (read 12 B per triangle of conn
    and 36 B of vertex positions, write 12 B per normal)."""
    for _ in range(3):
        tack.compute_normals(points, conn, n_pts, n_tris)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(reps):
        tack.compute_normals(points, conn, n_pts, n_tris)
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    nbytes = 48.0 * n_tris + 12.0 * n_pts
    return {"ms": ms, "gtris_per_s": n_tris / (ms * 1e-3) / 1e9,
            "algorithmic_gbs": nbytes / (ms * 1e-3) / 1e9,
            "note": "deterministic 64-bit fixed-point sums; includes one host sync (id check)"}


def time_soup(tack, torch, vol, grid, isos, cells, stream, reps=10):
    """tack_b200.algorithms.marching_cubes_soup on the same volume (count +
    unmerged soup + status check, device outputs): time per call (CUDA
    events; the call synchronises twice)."""
    iso = isos if len(isos) > 1 else isos[0]
    for _ in range(2):
        r = tack.algorithms.marching_cubes_soup(vol, grid, iso, copy_to_host=False)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(reps):
        r = tack.algorithms.marching_cubes_soup(vol, grid, iso, copy_to_host=False)
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    return {"ms": ms, "gcells_per_s": cells / (ms * 1e-3) / 1e9, "triangles": r["total_tris"],
            "output_gbs": 36.0 * r["total_tris"] / (ms * 1e-3) / 1e9}


def ctypes_f32(vals):
    import ctypes
    return (ctypes.c_float * len(vals))(*vals)


def run_e2e(args, tack, torch, dist, vol, grid, plan, eng, isos, world, rank, dev, cells):
    """Public API from pinned host memory: H2D volume, isosurface, D2H result."""
    host = torch.empty(vol.numel(), dtype=torch.float32, pin_memory=True)
    host.copy_(vol)
    dvol = torch.empty_like(vol)
    stream = torch.cuda.current_stream(dev)
    d2h = 0
    h2d = host.numel() * 4

    def once():
        nonlocal d2h
        if world == 1:
            # The public call on a pinned host tensor: H2D, filter, D2H.
            r = tack.flying_edges(host, grid, isos if len(isos) > 1 else isos[0])
            d2h = r["points"].nbytes + r["conn"].nbytes
        else:
            dvol.copy_(host, non_blocking=True)
            r = eng.run(dvol)
            p = torch.empty(r["points_field"].tensor.shape, dtype=torch.float32, pin_memory=True)
            c = torch.empty(r["conn_field"].tensor.shape, dtype=torch.int32, pin_memory=True)
            p.copy_(r["points_field"].tensor, non_blocking=True)
            c.copy_(r["conn_field"].tensor, non_blocking=True)
            stream.synchronize()
            d2h = p.numel() * 4 + c.numel() * 4
        return r

    def h2d_link_ms(reps=3):
        """Bare pinned host->device copy of the same bytes (the link bound)."""
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            dvol.copy_(host, non_blocking=True)
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    once()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.e2e_steps):
        once()
    t1.record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=dev)
    tot = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot)
    ms = float(ms.item())
    link = h2d_link_ms()
    return {"value": cells * args.e2e_steps / (ms * 1e-3) / 1e9, "unit": "Gcells/s",
            "h2d_bytes_per_step": int(tot[0].item()), "d2h_bytes_per_step": int(tot[1].item()),
            "ms_per_step": ms / args.e2e_steps, "steps": args.e2e_steps,
            "h2d_copy_alone_ms": link, "h2d_copy_alone_gbs": h2d / (link * 1e-3) / 1e9,
            "path": ("tack_b200.flying_edges(pinned host tensor): H2D of the volume, "
                     "count, emit, points/conn copied back into pinned numpy arrays"
                     if world == 1 else
                     "per rank: pinned H2D of its slab, SlabEngine.run, D2H of its slices")}


if __name__ == "__main__":
    sys.exit(main())
