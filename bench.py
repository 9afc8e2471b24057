#!/usr/bin/env python
"""Isosurface throughput on B200: input Gcells/s of flying-edges marching cubes.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tack_b200|reference]

Workload (default): 1024^3 f32 volume, sum of 32 seeded Gaussian blobs,
isovalue 0.5 -- the configuration the metric is quoted on at 1/2/4/8 GPUs.
The volume is z-slab sharded across N GPUs (one process per GPU, launched by
torchrun for N > 1): each rank classifies/counts/scans its slab, the
per-rank totals are exchanged on the device (by default one kernel storing
them into every rank's memory over NVLink, `--exchange nccl` for an NCCL
all-gather), each rank emits its slices of the single-volume output.  Total
work is fixed as N grows (strong scaling).  At N > 1 every rank's slices are
then compared, byte for byte, with the same rows of a single-GPU run of the
whole volume on rank 0 (`parity` in the JSON line).

A step = one isosurface of the whole volume from resident f32 values to
resident points + connectivity: classify, count + scan, the per-rank totals
exchanged on the device, device-side planning of the output bases, emit,
and an asynchronous copy of the totals to pinned host memory.  Output buffers
are allocated once, at this volume's exact size, from one host-planned run
before the timed steps (as when a caller processes a sequence of volumes);
every step's totals are checked against it afterwards.  `value` = cells of
the whole volume per second over K timed steps (CUDA events, max over ranks).  `e2e` = the same metric
through the public API from pinned host memory: each step copies the volume
host->device, runs flying_edges, copies points and connectivity back.

The reference arm (--impl reference) times the reference's own flying_edges
on its CPU backend (tack.cpu, llvmlite JIT, one thread per physical core),
imported from a copy of its Python sources in baseline/_ref
(`bench.py --install-reference <checkout>` makes the copy), on a bounded
sample of the same volume: a few z-slabs spread evenly over its depth.  The
C restatement of the same algorithm (the parity oracle) is timed beside it
on the same sample.  The GPU arm's cpu_baseline runs the same two legs on
the same sample.
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
    ap.add_argument("--cpu-steps", type=int, default=8,
                    help="timed steps of the reference leg of cpu_baseline (after 3 untimed)")
    ap.add_argument("--ref-backend", choices=["cpu", "cuda"], default="cpu",
                    help="--impl reference: the reference's tack.cpu (default) or its "
                         "tack.cuda backend (NVRTC kernels; the whole volume, one GPU)")
    ap.add_argument("--install-reference", metavar="CHECKOUT", default=None,
                    help="copy the reference's Python sources from a berkgeveci/tack "
                         "checkout into baseline/_ref and exit")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="totals exchange between ranks (N>1): NVLink peer stores or NCCL")
    ap.add_argument("--slabs", choices=["measured", "surface", "equal"], default="measured",
                    help="N>1: node-plane runs per rank: equal runs moved toward equal "
                         "measured device time per rank (default), runs balanced by the "
                         "surface of a first pass, or equal runs")
    ap.add_argument("--balance-slabs", action="store_true", help="the same as --slabs surface")
    args = ap.parse_args()
    if args.balance_slabs:
        args.slabs = "surface"
    return args


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
#
# The CPU legs time the reference's own flying edges (tack.cpu, its llvmlite
# JIT backend) and, beside it, the C port of the same algorithm (the parity
# oracle), on the same bounded sample of the workload: a few z-slabs spread
# evenly over the volume (so the surface's density along z is represented),
# every slab an independent flying_edges call on its own node planes.  The
# reference arm (--impl reference) and the GPU arm's cpu_baseline use the
# same sample and the same method, so they measure the same thing.

REF_DIR = os.path.join(REPO, "baseline", "_ref")
REF_TREES = (("tack-core", "src"), ("tack-vis", "src"))
CPU_SAMPLE_CELLS = 1.4e8   # cells per step of the CPU sample, all isovalues together
CPU_SAMPLE_SLABS = 8


def install_reference(checkout):
    """Copy the reference's pure-Python source trees (packages/tack-core/src,
    packages/tack-vis/src of a berkgeveci/tack checkout) into baseline/_ref,
    where the reference arm imports them from.  The reference's own build
    backend is not installable offline; the sources need no build."""
    import shutil
    for pkg, sub in REF_TREES:
        src = os.path.join(checkout, "packages", pkg, sub)
        dst = os.path.join(REF_DIR, pkg, sub)
        if not os.path.isdir(src):
            raise FileNotFoundError(src)
        if os.path.isdir(dst):
            shutil.rmtree(dst)
        shutil.copytree(src, dst, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    return REF_DIR


def load_reference_cpu():
    """The reference's tack on its CPU backend, imported from baseline/_ref.
    Returns (flying_edges, UniformGrid, field factory, f32 dtype, threads)."""
    paths = [os.path.join(REF_DIR, pkg, sub) for pkg, sub in REF_TREES]
    missing = [p for p in paths if not os.path.isdir(os.path.join(p, "tack"))]
    if missing:
        raise ImportError(f"no copy of the reference under {missing[0]} "
                          "(bench.install_reference copies it from a checkout)")
    for p in reversed(paths):
        if p not in sys.path:
            sys.path.insert(0, p)
    import tack as ref_tack
    from tack.runtime.dispatch import get_backend
    ref_tack.init(ref_tack.cpu)
    from tack.algorithms.flying_edges import UniformGrid, flying_edges
    return flying_edges, UniformGrid, ref_tack.field, ref_tack.f32, get_backend().num_threads


def cpu_sample_bounds(shape, niso):
    """Node-plane ranges [k0, k1) of the CPU sample: the whole volume when it
    is small, else CPU_SAMPLE_SLABS slabs centred at evenly spaced depths,
    their thickness set so a step is about CPU_SAMPLE_CELLS cells (all
    isovalues together), at least two cell layers each."""
    nx, ny, nz = shape
    per_plane = (nx - 1) * (ny - 1) * niso
    if per_plane * (nz - 1) <= CPU_SAMPLE_CELLS:
        return [(0, nz)]
    layers = int(max(2, round(CPU_SAMPLE_CELLS / (CPU_SAMPLE_SLABS * per_plane))))
    planes = min(nz, layers + 1)
    out = []
    for i in range(CPU_SAMPLE_SLABS):
        c = (2 * i + 1) * nz // (2 * CPU_SAMPLE_SLABS)
        k0 = min(max(0, c - planes // 2), nz - planes)
        out.append((k0, k0 + planes))
    return out


class CpuSample:
    """The slabs of the CPU sample as host f32 arrays (generated on the GPU
    when there is one)."""

    def __init__(self, config, shape, isos, device, volume=None):
        from tack_b200 import workloads
        self.shape, self.isos = shape, list(isos)
        self.bounds = cpu_sample_bounds(shape, len(self.isos))
        nx, ny, nz = shape
        self.slabs = []
        for k0, k1 in self.bounds:
            if volume is not None:  # the resident volume, planes [k0, k1)
                v = volume.view(nz, ny, nx)[k0:k1].reshape(-1).cpu().numpy()
            else:
                v = workloads.generate(config, shape, k0, k1, device=device).cpu().numpy()
            self.slabs.append((k0, k1, v))
        self.cells = sum((nx - 1) * (ny - 1) * (k1 - k0 - 1) for k0, k1 in self.bounds)

    def describe(self):
        nx, ny, nz = self.shape
        if self.bounds == [(0, nz)]:
            where = "the whole volume"
        else:
            where = ", ".join(f"[{a},{b})" for a, b in self.bounds)
            where = f"node planes {where}"
        return (f"{where} of the {nx}x{ny}x{nz} volume: {self.cells} cells per isovalue, "
                f"one flying_edges call per slab and isovalue per step")


def time_reference_cpu(sample, steps, warmup):
    """Per-step seconds of the reference's tack.cpu flying_edges over the
    sample (fields created once, outside the timing, as resident inputs)."""
    fe, Grid, field, f32, threads = load_reference_cpu()
    nx, ny, _ = sample.shape
    calls = []
    for k0, k1, v in sample.slabs:
        f = field(dtype=f32, shape=(v.size,))
        f.from_numpy(v)
        calls.append((f, Grid(nx - 1, ny - 1, k1 - k0 - 1, 0.0, 0.0, float(k0), 1.0, 1.0, 1.0)))

    def step():
        t0 = time.perf_counter()
        for f, g in calls:
            for iso in sample.isos:
                fe(f, g, iso)
        return time.perf_counter() - t0

    for _ in range(warmup):
        step()
    return [step() for _ in range(steps)], threads


def time_port_cpu(sample, steps, warmup):
    """Per-step seconds of the C port (the parity oracle, pthreads over rows,
    every host thread) over the sample."""
    from oracle import oracle
    oracle.build()
    nthreads = oracle.num_threads(0)
    nx, ny, _ = sample.shape
    calls = [(v, oracle.Grid(nx - 1, ny - 1, k1 - k0 - 1, 0.0, 0.0, float(k0), 1.0, 1.0, 1.0))
             for k0, k1, v in sample.slabs]

    def step():
        t0 = time.perf_counter()
        for v, g in calls:
            oracle.flying_edges_isovalues(v, g, sample.isos, nthreads=nthreads)
        return time.perf_counter() - t0

    for _ in range(warmup):
        step()
    return [step() for _ in range(steps)], nthreads


def host_cores():
    """Physical cores and the CPU model of this host (from lscpu)."""
    info = {"logical": os.cpu_count()}
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        kv = dict(line.split(":", 1) for line in out.splitlines() if ":" in line)
        kv = {k.strip(): v.strip() for k, v in kv.items()}
        info["model"] = kv.get("Model name")
        sockets = int(kv.get("Socket(s)", "1") or 1)
        cores = int(kv.get("Core(s) per socket", "0") or 0)
        if cores:
            info["physical"] = sockets * cores
    except (OSError, ValueError, subprocess.SubprocessError):
        pass
    return info


def cpu_legs(sample, steps, warmup, port_steps=3):
    """Both CPU legs on the sample: the reference's tack.cpu (kind
    "reference"; the port alone, kind "port", when the reference cannot be
    imported here) and the C port beside it.  Each leg's value is the cells
    of the sample (times the isovalues) over the median step time.  Returns
    the cpu_baseline dict."""
    cores = host_cores()
    legs = {}
    try:
        t, threads = time_reference_cpu(sample, steps, warmup)
        legs["reference"] = {"value": sample.cells * len(sample.isos) / statistics.median(t) / 1e9,
                             "cores": threads, "kind": "reference",
                             "seconds_per_step": statistics.median(t), "steps": len(t),
                             "what": "the reference's flying_edges on tack.cpu (llvmlite JIT), "
                                     "imported from its source tree in baseline/_ref, "
                                     "TACK_CPU_THREADS unset (one thread per physical core)"}
    except Exception as e:  # the reference could not be imported or run here
        legs["reference_error"] = f"{type(e).__name__}: {e}"
    t, nthreads = time_port_cpu(sample, port_steps, 1)
    legs["port"] = {"value": sample.cells * len(sample.isos) / statistics.median(t) / 1e9,
                    "cores": nthreads, "kind": "port", "seconds_per_step": statistics.median(t),
                    "steps": len(t),
                    "what": "the C restatement of the reference's kernels and host "
                            "orchestration (the parity oracle), pthreads over rows"}
    head = legs.get("reference") or legs["port"]
    out = {"value": head["value"], "unit": "Gcells/s", "cores": head["cores"],
           "kind": head["kind"], "sample": sample.describe(), "host_cores": cores}
    out.update(legs)
    return out


def run_reference_cuda(args, local):
    """The reference's flying_edges on its own CUDA backend (tack.cuda: NVRTC
    kernels, one thread per row, host prefix sums between the passes) over
    the whole volume on this GPU; each call as the reference makes it (its
    zero mask filled on the host and copied in, the row arrays copied out and
    summed on the host, the result copied back to numpy)."""
    import torch
    from tack_b200 import workloads
    cfg = workloads.CONFIGS[args.config]
    shape = tuple(args.size) if args.size else cfg["shape"]
    nx, ny, nz = shape
    vol = workloads.generate(args.config, shape, device=torch.device("cuda", local))
    host = vol.cpu().numpy()
    del vol
    torch.cuda.synchronize()
    paths = [os.path.join(REF_DIR, pkg, sub) for pkg, sub in REF_TREES]
    for p in reversed(paths):
        if p not in sys.path:
            sys.path.insert(0, p)
    import tack as ref_tack
    ref_tack.init(ref_tack.cuda)
    from tack.algorithms.flying_edges import UniformGrid, flying_edges
    f = ref_tack.field(dtype=ref_tack.f32, shape=(host.size,))
    f.from_numpy(host)
    g = UniformGrid(nx - 1, ny - 1, nz - 1, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
    cells = (nx - 1) * (ny - 1) * (nz - 1)

    def call():
        t0 = time.perf_counter()
        out = None
        for iso in cfg["isovalues"]:
            out = flying_edges(f, g, iso)
        return time.perf_counter() - t0, out

    for _ in range(max(1, args.warmup)):
        call()
    times = []
    out = None
    for _ in range(args.steps):
        t, out = call()
        times.append(t)
    t = statistics.median(times)
    value = cells / t / 1e9
    line = {
        "impl": "reference", "backend": "tack.cuda", "metric": METRIC, "value": value,
        "unit": "Gcells/s", "n_gpus": 1, "steps": args.steps, "warmup": max(1, args.warmup),
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args.config, shape, cfg["isovalues"]),
                   "volume_nodes": list(shape), "isovalues": cfg["isovalues"]},
        "outputs": {"points": int(out["total_points"]) if out else 0,
                    "triangles": int(out["total_tris"]) if out else 0},
        "e2e": {"value": value, "unit": "Gcells/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": ("the reference's own GPU path: flying_edges on tack.cuda from baseline/_ref, "
                 "the volume resident in a tack field, median wall time of whole calls"),
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    if args.ref_backend == "cuda":
        return run_reference_cuda(args, local)
    import torch
    from tack_b200 import workloads
    cfg = workloads.CONFIGS[args.config]
    shape = tuple(args.size) if args.size else cfg["shape"]
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    sample = CpuSample(args.config, shape, cfg["isovalues"], device)
    # JIT compilation takes the first calls: at least three untimed steps.
    base = cpu_legs(sample, args.steps, max(3, args.warmup))
    head = base.get("reference") or base["port"]
    value = head["value"]
    ms = head["seconds_per_step"] * 1e3
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "Gcells/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args.config, shape, cfg["isovalues"]),
                   "volume_nodes": list(shape), "isovalues": cfg["isovalues"],
                   "sample": sample.describe()},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": "Gcells/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": ("host cores only; value = cells of the sample x isovalues per second of "
                 "the reference's own flying_edges on tack.cpu (kind 'reference'), or of "
                 "the C port when the reference cannot be imported (kind 'port')"),
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
    if args.install_reference:
        print(install_reference(args.install_reference))
        return 0
    if args.impl == "reference":
        return run_reference(args)
    import torch
    import torch.distributed as dist

    import tack_b200 as tack
    from tack_b200 import _lib, workloads
    from tack_b200.distributed import (SlabEngine, SlabPlan, balanced_bounds,
                                       rebalanced_bounds, slab_bases)

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
    grid = tack.UniformGrid(nxn - 1, nyn - 1, nzn - 1, 0.0, 0.0, 0.0, 1.0, 1.0, 1.0)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    niso = len(isos)
    isoc = (ctypes_f32(isos))
    cells = (nxn - 1) * (nyn - 1) * (nzn - 1)
    counts_host = torch.zeros(niso * 4, dtype=torch.int64, pin_memory=True)
    K = args.steps
    KP = min(K, 50)

    def setup(bounds):
        """This rank's slab on `bounds` (None: equal runs): its volume, engine,
        one host-planned run, and output buffers of its exact size; the timed
        steps then run count -> plan -> emit with no host round trip (the
        totals reach the host asynchronously, as a caller would read them)."""
        plan = SlabPlan(nzn, world, rank, bounds=bounds)
        vol = workloads.generate(args.config, shape, plan.k0, plan.k1, device=dev)
        torch.cuda.synchronize()
        eng = SlabEngine(grid, plan, isos, exchange=args.exchange)
        first = eng.run(vol)
        own = first["counts"]
        own_p, own_t = int(own[:, :3].sum()), int(own[:, 3].sum())
        pts_buf = torch.empty(max(own_p, 1) * 3, dtype=torch.float32, device=dev)
        conn_buf = torch.empty(max(own_t, 1) * 3, dtype=torch.int32, device=dev)
        return plan, vol, eng, first, pts_buf, conn_buf

    def phases(eng, vol, pts_buf, conn_buf):
        """Warm-up steps, then phase times: CUDA events between the phases of
        KP ordinary (not graph) steps (ms: threshold, count, totals exchange /
        plan, emit); the headline time is measured separately."""
        for _ in range(args.warmup):
            eng.run_device(vol, pts_buf, conn_buf, counts_host)
        ev = {k: [torch.cuda.Event(enable_timing=True) for _ in range(KP)] for k in "abcde"}
        for i in range(KP):
            eng.run_device(vol, pts_buf, conn_buf, counts_host, [ev[k][i] for k in "abcde"])
        torch.cuda.synchronize()

        def mean(a, b):
            return sum(ev[a][i].elapsed_time(ev[b][i]) for i in range(KP)) / KP
        return mean("a", "b"), mean("b", "c"), mean("c", "d"), mean("d", "e")

    balanced = None
    plan, vol, eng, first, pts_buf, conn_buf = setup(None)
    if world > 1 and args.slabs == "surface":
        # Slab bounds balanced by predicted device time: the surface of this
        # first pass (in a time series, the previous step's) gives each node
        # plane's triangles; a plane costs NODE_COST per node (the threshold
        # read) plus TRI_COST per triangle (count and emit).  Then the slabs
        # are set up again on the new bounds.
        tris = eng.plane_triangles(first["counts"])
        allt = [None] * world
        dist.all_gather_object(allt, tris.tolist())
        plane_tris = np.concatenate([np.asarray(t, np.float64) for t in allt])
        work = NODE_COST * nxn * nyn + TRI_COST * plane_tris
        balanced = balanced_bounds(work, world)
        eng.close()
        del eng, vol, first, pts_buf, conn_buf
        plan, vol, eng, first, pts_buf, conn_buf = setup(balanced)
    k1, k2, host, k3 = phases(eng, vol, pts_buf, conn_buf)
    moves = []
    if world > 1 and args.slabs == "measured":
        # Bounds moved toward equal device time per rank, from every rank's
        # measured threshold + count + emit time on the current bounds (the
        # exchange wait left out), at most twice; every rank gets the same
        # gathered times, so all take the same decision.
        for _ in range(2):
            t = torch.tensor([k1, k1 + k2 + k3, float(plan.p0), float(plan.p1)],
                             dtype=torch.float64, device=dev)
            allt = [torch.zeros_like(t) for _ in range(world)]
            dist.all_gather(allt, t)
            allt = np.stack([a.cpu().numpy() for a in allt])
            cur = [int(x) for x in allt[:, 2]] + [int(allt[-1, 3])]
            new = rebalanced_bounds(cur, allt[:, 0], allt[:, 1])
            if max(abs(a - b) for a, b in zip(new, cur)) <= 1:
                break
            moves.append({"bounds": cur, "busy_ms": [round(float(x), 4) for x in allt[:, 1]]})
            balanced = new
            eng.close()
            del eng, vol, first, pts_buf, conn_buf
            plan, vol, eng, first, pts_buf, conn_buf = setup(balanced)
            k1, k2, host, k3 = phases(eng, vol, pts_buf, conn_buf)
    local_nodes = vol.numel()
    own = first["counts"]
    own_p, own_t = int(own[:, :3].sum()), int(own[:, 3].sum())
    bases = first["bases"]

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
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
    # Every rank's phase times, so the slowest rank and the time the others
    # spend waiting for it in the exchange are visible.
    mine = torch.tensor([ms, k1, k2, host, k3, float(own_p), float(own_t)], dtype=torch.float64,
                        device=dev)
    per_rank = [mine]
    if world > 1:
        per_rank = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(per_rank, mine)
    per_rank = np.stack([t.cpu().numpy() for t in per_rank])
    ms, k1, k2, host, k3 = (float(x) for x in per_rank[:, :5].max(axis=0))
    total_points = int(bases["totals"][:, 0].sum())
    total_tris = int(bases["totals"][:, 1].sum())
    ranks = None
    if world > 1:
        arrive = per_rank[:, 1] + per_rank[:, 2]  # threshold + count: ready to exchange
        ranks = {
            "k1_threshold_ms": [round(float(x), 4) for x in per_rank[:, 1]],
            "k2_count_scan_ms": [round(float(x), 4) for x in per_rank[:, 2]],
            "exchange_plan_ms": [round(float(x), 4) for x in per_rank[:, 3]],
            "k3_emit_ms": [round(float(x), 4) for x in per_rank[:, 4]],
            "points": [int(x) for x in per_rank[:, 5]],
            "triangles": [int(x) for x in per_rank[:, 6]],
            "slowest_to_exchange": int(np.argmax(arrive)),
            "arrival_skew_ms": round(float(arrive.max() - arrive.min()), 4),
            "exchange_wait_spread_ms": round(float(per_rank[:, 3].max() - per_rank[:, 3].min()), 4),
            "note": ("phase means over ordinary (not graph) steps on each rank; a rank's "
                     "exchange_plan time is mostly its wait for the last rank to arrive, so "
                     "the spread of those times is the arrival skew seen on the device"),
        }

    # ---- parity of the timed path's output (outside the timed region) -----
    parity = check_parity(args, tack, torch, dist, shape, isos, grid, first["all_counts"],
                          pts_buf, conn_buf, world, rank, dev)

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

    # ---- CPU baseline (host cores), N == 1 only: the same sample and method
    # as the reference arm (bench.py --impl reference) ----------------------
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        sample = CpuSample(args.config, shape, isos, dev, volume=vol)
        cpu = cpu_legs(sample, args.cpu_steps, 3)

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
                                f"{slab_words(args.slabs, balanced)})"
                                if world > 1 else "single GPU"),
                "slab_bounds": balanced,
                "slab_moves": moves or None,
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
                           "totals_gather_plan": host, "k3_emit": k3,
                           "note": "each phase's max over ranks"},
            "per_rank": ranks,
            "parity": parity,
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


def slab_words(mode, bounds):
    """How the node planes were split, for the JSON line."""
    if bounds is None:
        return "equal plane runs"
    if mode == "surface":
        return "plane runs balanced by surface"
    return "plane runs moved toward equal measured device time per rank"


def check_parity(args, tack, torch, dist, shape, isos, grid, all_counts, pts_buf, conn_buf,
                 world, rank, dev):
    """Every rank's output slices from the timed path (the last graph replay)
    against the same rows of one single-GPU flying_edges call on the whole
    volume, run on rank 0: points compared as bit patterns, conn exactly.
    Ranks send their slices to rank 0 (NCCL point-to-point); every rank
    raises if any slice differs.  Outside the timed region."""
    from tack_b200 import workloads
    from tack_b200.distributed import slab_bases
    allc = np.asarray(all_counts, np.int64)  # [world, niso, 4]
    niso = allc.shape[1]
    sizes = [(int(allc[r, :, :3].sum()), int(allc[r, :, 3].sum())) for r in range(world)]
    ok = torch.ones(1, dtype=torch.int32, device=dev)
    checked_pts = checked_tris = 0
    info = {}
    if rank == 0:
        nx, ny, nz = shape
        whole = workloads.generate(args.config, shape, 0, nz, device=dev)
        ref = tack.flying_edges(whole, grid, isos if len(isos) > 1 else isos[0],
                                copy_to_host=False)
        del whole
        ref_p = ref["points_field"].tensor.view(torch.int32).view(-1, 3)
        ref_c = ref["conn_field"].tensor.view(-1, 3)
        P_all, T_all = ref["total_points"], ref["total_tris"]
        good = (P_all == int(allc[:, :, :3].sum())) and (T_all == int(allc[:, :, 3].sum()))
        for r in range(world):
            P, T = sizes[r]
            if r == 0:
                p = pts_buf[:P * 3]
                c = conn_buf[:T * 3]
            else:
                p = torch.empty(P * 3, dtype=torch.float32, device=dev)
                c = torch.empty(T * 3, dtype=torch.int32, device=dev)
                if P:
                    dist.recv(p, src=r)
                if T:
                    dist.recv(c, src=r)
            p = p.view(torch.int32).view(-1, 3)
            c = c.view(-1, 3)
            b = slab_bases(allc, r)
            for q in range(niso):
                for sct in range(3):
                    n = int(allc[r, q, sct])
                    lo, go = int(b["out_base"][q, sct]), int(b["pt_global_out"][q, sct])
                    good &= bool(torch.equal(p[lo:lo + n], ref_p[go:go + n]))
                    checked_pts += n
                n = int(allc[r, q, 3])
                lo, go = int(b["tri_out"][q]), int(b["tri_global"][q])
                good &= bool(torch.equal(c[lo:lo + n], ref_c[go:go + n]))
                checked_tris += n
        good &= checked_pts == P_all and checked_tris == T_all
        ok.fill_(1 if good else 0)
        info = {"points": P_all, "triangles": T_all, "points_checked": checked_pts,
                "triangles_checked": checked_tris}
        del ref, ref_p, ref_c
    else:
        P, T = sizes[rank]
        if P:
            dist.send(pts_buf[:P * 3].contiguous(), dst=0)
        if T:
            dist.send(conn_buf[:T * 3].contiguous(), dst=0)
    if world > 1:
        dist.broadcast(ok, src=0)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if int(ok.item()) != 1:
        raise RuntimeError("parity: the timed path's output differs from the single-GPU "
                           "flying_edges of the whole volume")
    info.update({"checked": True, "ranks_equal": world,
                 "against": "one single-GPU tack_b200.flying_edges call on the whole volume "
                            "(rank 0); points bit for bit, conn exact, every row once"})
    return info


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
