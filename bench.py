#!/usr/bin/env python
"""Throughput of the permutohedral-lattice filter, forward + backward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = forward + value-gradient backward of one 1024x1024 image, pd = 5
(x/32, y/32, rgb/0.08 of a seeded 200-cell Voronoi image), vd = 3, through
the public autograd API (PermutoLatticeFunction).  Each rank of a torchrun
job filters its own image(s) (weak scaling, no collective on the data path);
``value`` is all pixels of all ranks over the slowest rank's device time.

``--impl ours`` (default) times this repository's sm_100a library;
``--impl reference`` times the reference CUDA extension (PLOO, built from the
reference sources for sm_100a into oracle/_ref) through its own forward /
backward with the same protocol, on rank 0 only.

Timing: W untimed warm-up steps, then exactly K steps, each bracketed by CUDA
events on the launching stream; L2 is flushed (256 MiB write) between steps,
outside the events.  ``e2e`` repeats the K steps from pinned host buffers:
H2D of features/values/grad and D2H of out/grad inside the timed region, the
copies on their own streams so that they overlap the kernels of neighbouring
steps (the same pipeline for both arms).  Prints one JSON line (rank 0).
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "Mpixel/s fwd+bwd (1024², pd=5, vd=3) at 1/2/4/8 B200; % of HBM roofline"
UNIT = "Mpixel/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="voronoi1024_pd5_vd3")
    ap.add_argument("--images-per-gpu", type=int, default=1)
    ap.add_argument("--batch-split", type=int, default=0,
                    help="a fixed batch of this many images of the workload, split by image over the "
                         "ranks (shard_range), one batch call per rank and step (strong scaling); the "
                         "reference arm loops over the whole batch on one GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample", type=int, default=2048, help="output pixels of the CPU sample")
    ap.add_argument("--profile-steps", type=int, default=10)
    ap.add_argument("--soak-seconds", type=float, default=1.0,
                    help="untimed steps before warm-up so that clocks settle under load")
    ap.add_argument("--mode", choices=["full", "device"], default="full",
                    help="device: only the warm-up and the K device-timed steps (for profilers)")
    ap.add_argument("--batched", action="store_true",
                    help="ours: the images of a rank go through one batch call per step "
                         "(PermutoLatticeBatchFunction) instead of one call per image")
    ap.add_argument("--feature-grad", action="store_true",
                    help="time forward + backward with the feature gradient as well "
                         "(PermutoLatticeFeatureFunction) next to the value gradient only; 1 GPU, ours only")
    ap.add_argument("--kept-lattice", action="store_true",
                    help="time filter forward + backward on a lattice built once (a mean-field "
                         "iteration), next to the full forward + backward; 1 GPU, ours only")
    ap.add_argument("--lattice-precision", choices=["fp32", "bf16"], default="fp32",
                    help="ours: lattice rows of the blur's streaming passes (large lattices) in float "
                         "or bfloat16 (PLOO.set_lattice_precision; off by default)")
    return ap.parse_args()


# ---------------------------------------------------------------- distributed plumbing

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    if local_world > 1:   # each rank its own share of the host cores (the host enqueues every launch)
        cpus = sorted(os.sched_getaffinity(0))
        per = max(1, len(cpus) // local_world)
        mine = cpus[local * per:(local + 1) * per] or cpus
        try:
            os.sched_setaffinity(0, mine)
            torch.set_num_threads(len(mine))
        except OSError:
            pass
    torch.cuda.set_device(local)
    return rank, world, local


def dist_init(world, local):
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))


def barrier(world):
    from plattice_pytorch_b200.sharding import barrier as _barrier
    _barrier(world)


def max_over_ranks(x, world):
    from plattice_pytorch_b200.sharding import max_over_ranks as _max
    return _max(x, world, device="cuda")


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi sampling of the clocks and throttle reasons of the given GPUs
    (one sampler process per node: local rank 0 samples every rank's GPU, so
    that N ranks do not start N nvidia-smi processes on the host cores that
    enqueue their launches)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, devices):
        self.proc = None
        self.path = None
        sel = []
        try:
            ids = []
            for d in devices:
                p = torch.cuda.get_device_properties(d)
                ids.append(f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0")
            sel = ["-i", ",".join(ids)]
        except Exception:
            sel = []
        self.gpus = len(devices)
        self.cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                    "-lms", "100"] + sel

    def start(self):
        import tempfile
        fd, self.path = tempfile.mkstemp(prefix="plattice_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(self.cmd, stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        rows = []
        with open(self.path) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        pw = [num(r[3]) for r in rows if num(r[3]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        top = max(mx) if mx else None
        loaded = [s for s in sm if top and s >= 0.5 * top] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": top,
                "power_w_max": max(pw) if pw else None, "samples": len(rows), "gpus": self.gpus,
                "reasons": reasons}


# ---------------------------------------------------------------- implementations

def ours_impl():
    from plattice_pytorch_b200 import PermutoLatticeFunction, _lib
    _lib.lib()   # the CUDA library must load: there is no fallback
    return PermutoLatticeFunction


def reference_impl():
    from oracle import ref as oref
    if not oref.ploo_available():
        return None, "reference extension not built (make -C oracle ref)"
    P = oref.load_ploo()

    class RefFunction(torch.autograd.Function):
        """The reference's own plattice.py Function (plattice.py:7-19) over its PLOO."""

        @staticmethod
        def forward(ctx, feature, values):
            weight, out = P.forward(feature, values)
            ctx.save_for_backward(weight, feature)
            return out

        @staticmethod
        @torch.autograd.function.once_differentiable
        def backward(ctx, grad_output):
            weight, feature = ctx.saved_tensors
            return None, P.backward(feature, grad_output.contiguous(), weight)

    return RefFunction, None


def step(fn, f, v, g):
    out = fn.apply(f, v)
    (gv,) = torch.autograd.grad(out, (v,), (g,))
    return out, gv


# ---------------------------------------------------------------- measurement

def load_inputs(args, rank, world):
    """This rank's images: `images_per_gpu` of its own (weak scaling), or its
    contiguous share of a fixed batch of `batch_split` images (strong)."""
    from plattice_pytorch_b200.sharding import shard_range
    from plattice_pytorch_b200.workloads import make_workload
    if args.batch_split:
        start, stop = shard_range(args.batch_split, world, rank)
        return [make_workload(args.workload, seed=i, index=i) for i in range(start, stop)]
    return [make_workload(args.workload, seed=rank * args.images_per_gpu + i)
            for i in range(args.images_per_gpu)]


def timed_device(fn, batch, steps, flush, host_us=None):
    """Per-step CUDA-event time (ms) summed over `steps`; L2 flushed between
    steps.  With `host_us` (a list), also the host time of each step's
    enqueue (the library and autograd calls, no synchronisation), in us."""
    evs = []
    for _ in range(steps):
        flush.fill_(1.0)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        t0 = time.perf_counter()
        for (f, v, g) in batch:
            step(fn, f, v, g)
        if host_us is not None:
            host_us.append((time.perf_counter() - t0) * 1e6)
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    per = [a.elapsed_time(b) for a, b in evs]
    if host_us is None:
        return sum(per)
    return per


def kept_lattice_line(args, dev):
    """One JSON line: filter forward + value-gradient backward on a kept lattice
    (LatticeFilterFunction), per step, against the full forward + backward
    (PermutoLatticeFunction, lattice rebuilt every step); L2 flushed between
    steps, CUDA events on the launching stream."""
    from plattice_pytorch_b200 import PLOO, LatticeFilterFunction, PermutoLatticeFunction
    from plattice_pytorch_b200.workloads import make_workload
    wl = make_workload(args.workload, seed=0)
    f = torch.from_numpy(wl["features"]).to(dev)
    v = torch.from_numpy(wl["values"]).to(dev).requires_grad_(True)
    g = torch.from_numpy(wl["grad"]).to(dev)
    h, w, pd = f.shape
    _, _, lat = PLOO.lattice_forward(f, v.detach())

    class Kept:   # the step() protocol over the kept lattice
        @staticmethod
        def apply(ff, vv):
            return LatticeFilterFunction.apply(vv, lat)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    res = {}
    for name, fn in (("kept", Kept), ("full", PermutoLatticeFunction)):
        for _ in range(args.warmup):
            step(fn, f, v, g)
        res[name] = timed_device(fn, [(f, v, g)], args.steps, flush) / args.steps
    n = h * w
    return {"metric": "Mpixel/s filter fwd+bwd on a kept lattice (mean-field iteration)",
            "value": n / (res["kept"] * 1e-3) / 1e6, "unit": "Mpixel/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["kept"], "higher_is_better": True,
            "full_ms_per_step": res["full"], "speedup_vs_rebuild": res["full"] / res["kept"],
            "lattice": PLOO.lattice_info(lat), "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "h": int(h), "w": int(w), "pd": int(pd),
                       "vd": int(v.shape[2]), "l2": "flushed between timed steps"}}


def feature_grad_line(args, dev):
    """One JSON line: forward + backward for both inputs (features and values)
    per step, against forward + value gradient only; L2 flushed between
    steps, CUDA events on the launching stream."""
    from plattice_pytorch_b200 import PermutoLatticeFeatureFunction, PermutoLatticeFunction
    from plattice_pytorch_b200.workloads import make_workload
    wl = make_workload(args.workload, seed=0)
    f = torch.from_numpy(wl["features"]).to(dev).requires_grad_(True)
    v = torch.from_numpy(wl["values"]).to(dev).requires_grad_(True)
    g = torch.from_numpy(wl["grad"]).to(dev)
    h, w, pd = f.shape
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def both():
        out = PermutoLatticeFeatureFunction.apply(f, v)
        torch.autograd.grad(out, (f, v), (g,))

    def values_only():
        out = PermutoLatticeFunction.apply(f.detach(), v)
        torch.autograd.grad(out, (v,), (g,))

    res = {}
    for name, fn in (("both", both), ("values", values_only)):
        for _ in range(args.warmup):
            fn()
        evs = []
        for _ in range(args.steps):
            flush.fill_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
        res[name] = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    n = h * w
    return {"metric": "Mpixel/s fwd + bwd with feature and value gradients",
            "value": n / (res["both"] * 1e-3) / 1e6, "unit": "Mpixel/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["both"], "higher_is_better": True,
            "value_grad_only_ms_per_step": res["values"], "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "h": int(h), "w": int(w), "pd": int(pd),
                       "vd": int(v.shape[2]), "l2": "flushed between timed steps"}}


RING = 3   # steps of the end-to-end pipeline in flight


def timed_e2e(fn, host, steps, dev):
    """Whole-loop CUDA-event time (ms) of `steps` end-to-end steps from pinned
    host buffers, including H2D of the inputs (features, values, upstream
    gradient) and D2H of the step's result, the value gradient.  The forward
    output stays on the device, where it feeds the loss that the upstream
    gradient stands for.

    The same pipeline serves both arms: each step's inputs are copied in on an
    input stream, the filter runs on the default stream (where the reference
    launches its kernels whatever the current stream is), and the gradient is
    copied back on an output stream, with events ordering the three.  The two
    copy directions and the kernels of different steps overlap; every step
    still moves its own inputs and result."""
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    comp = torch.cuda.default_stream(dev)
    outs = [[torch.empty(h[1].shape, pin_memory=True) for h in host] for _ in range(RING)]
    # device input buffers of RING steps (and host result buffers), reused once
    # the step that used them has finished; the host waits for that step
    # before reusing its slot, so it runs at most RING steps ahead (a bounded
    # queue, as in a serving loop, and no allocator growth inside the timed loop)
    dins = [[tuple(torch.empty(x.shape, dtype=x.dtype, device=dev) for x in hh) for hh in host]
            for _ in range(RING)]
    freed = [None] * RING
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    for i in range(steps):
        r = i % RING
        if freed[r] is not None:
            freed[r].synchronize()
        for k, (hf, hv, hg) in enumerate(host):
            hgr = outs[r][k]
            f, v, g = dins[r][k]
            with torch.cuda.stream(s_in):
                f.copy_(hf, non_blocking=True)
                v.copy_(hv, non_blocking=True)
                g.copy_(hg, non_blocking=True)
            comp.wait_stream(s_in)
            with torch.cuda.stream(comp):
                out, gv = step(fn, f, v.detach().requires_grad_(True), g)
            s_out.wait_stream(comp)
            gv.record_stream(s_out)
            with torch.cuda.stream(s_out):
                hgr.copy_(gv, non_blocking=True)
        freed[r] = torch.cuda.Event()
        freed[r].record(s_out)   # the step's inputs are read and its result copied out
    comp.wait_stream(s_in)
    comp.wait_stream(s_out)
    e1.record(comp)
    e1.synchronize()
    return e0.elapsed_time(e1)


def graph_stats(impl):
    """(captures, replays) of the library's call graphs so far ((0, 0) for the reference)."""
    if impl != "ours":
        return 0, 0
    from plattice_pytorch_b200 import PLOO
    return PLOO.graph_cache_stats()


def hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def kernel_bytes(stage, n, pd, vd, m, u, cap_log2):
    """Compulsory HBM bytes per step of a stage of this implementation (reads
    + writes of the data it must touch once; L2-resident gathers not
    counted)."""
    K = pd + 1
    CW = (4 + 2 * pd + 15) // 16
    pad = (lambda c: c if c <= 2 else ((c + 3) // 4) * 4)
    CPF, CPB = pad(vd + 1), pad(vd)
    slot = 6 * K * n   # uint16 local id + float weight per slot
    per = {
        "tile_build": n * 4 * pd + slot + u * (16 * CW + 4 * CPF),
        "clear": (1 << cap_log2) * (5 if cap_log2 >= 22 else 4),   # cells, + the miss filter's byte per cell
        "insert": u * (2 * 16 * CW + 8) + m * (2 * 16 * CW + 8),   # insert + compaction
        "splat_fwd": slot + n * 4 * vd + m * 4 * CPF,
        "neighbors": m * (16 * CW + 8 * K),
        "blur_fwd": K * m * (8 * CPF + 8),
        "slice_fwd": slot + m * 4 * CPF + n * 4 * (vd + 1),
        "zero": m * 4 * CPB,
        "splat_bwd": slot + n * 4 * (vd + 1) + m * 4 * CPB,
        "blur_bwd": K * m * (8 * CPB + 8),
        "slice_bwd": slot + m * 4 * CPB + n * 4 * vd,
    }
    return per[stage]


def stage_bytes(n, pd, vd, m):
    """Algorithmic bytes of splat + blur + slice (lattice build excluded):
    B_fwd = N(8V+16K+4) + M(8(V+1)(K+1) + 8K), B_bwd = N(8V+16K+4) + M(8V(K+1) + 8K)."""
    K = pd + 1
    b_fwd = n * (8 * vd + 16 * K + 4) + m * (8 * (vd + 1) * (K + 1) + 8 * K)
    b_bwd = n * (8 * vd + 16 * K + 4) + m * (8 * vd * (K + 1) + 8 * K)
    return b_fwd, b_bwd


def profile_ours(fn, batch, steps, flush, batched, groups=False):
    """Per-stage device times from CUDA events around every launch (untimed
    run) of the first image (or of the batch, for a batch call); with
    `groups`, events around the launch groups only (build, forward filter,
    backward filter)."""
    from plattice_pytorch_b200 import PLOO, _lib
    f, v, g = batch[0]
    if batched:
        _, _, lat = PLOO.batch_forward(f, v.detach())
    else:
        _, _, lat = PLOO.lattice_forward(f, v.detach())
    info = PLOO.lattice_info(lat)
    del lat
    _lib.profile_read()
    _lib.profile_enable(True, groups=groups)
    try:
        for _ in range(steps):
            flush.fill_(1.0)
            step(fn, f, v, g)
        torch.cuda.synchronize()
        prof = _lib.profile_read()
    finally:
        _lib.profile_enable(False)
    return info, prof


def traffic_from_profiles(kernel):
    """ncu DRAM bytes per launch recorded for `kernel` in profiles/traffic.txt
    ('<stage> <bytes per launch>' lines), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    try:
        with open(path) as fh:
            for line in fh:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == kernel:
                    return float(parts[1])
    except OSError:
        pass
    return None


def atomics_from_profiles():
    """ncu reduction / CAS request counts per launch recorded in profiles/atomics.txt."""
    path = os.path.join(ROOT, "profiles", "atomics.txt")
    out = {}
    try:
        with open(path) as fh:
            for line in fh:
                parts = line.split()
                if len(parts) >= 2 and not line.startswith("#"):
                    out[parts[0]] = int(parts[1])
    except OSError:
        pass
    return out


def cpu_baseline(f_np, v_np, g_np, sample):
    """The brute-force dense Gaussian (oracle port of the reference test's
    brute_force_bilateral, generalised) on `sample` output pixels forward and
    `sample` backward, all host threads."""
    import oracle
    threads = len(os.sched_getaffinity(0))
    n = f_np.shape[0] * f_np.shape[1]
    rows = range(0, min(sample, n))
    t0 = time.perf_counter()
    oracle.brute_gaussian(f_np, v_np, rows=rows, threads=threads)
    t1 = time.perf_counter()
    wt = np.full(n, 1.0 / n, np.float32)
    oracle.brute_gaussian(f_np, g_np, rows=rows, threads=threads, weight=wt)
    t2 = time.perf_counter()
    px = rows.stop - rows.start
    cpu = "unknown"
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    cpu = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"value": px / (t2 - t0) / 1e6, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"brute-force O(N^2) Gaussian: {px} output pixels forward + {px} backward "
                      f"of the {n}-pixel image ({t1 - t0:.2f} s + {t2 - t1:.2f} s)",
            "cpu": cpu}


def cpu_lattice_oracle(f_np, v_np, g_np):
    """The sequential C restatement of the lattice filter on one core (whole image)."""
    import oracle
    t0 = time.perf_counter()
    wo, _, _ = oracle.forward(f_np, v_np)
    oracle.backward(f_np, g_np, wo)
    dt = time.perf_counter() - t0
    n = f_np.shape[0] * f_np.shape[1]
    return {"value": n / dt / 1e6, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"lattice oracle, whole image forward + backward ({dt:.2f} s)"}


def main():
    args = parse_args()
    rank, world, local = dist_setup()
    dev = torch.device("cuda", local)

    if args.feature_grad:
        if rank == 0 and args.impl == "ours":
            print(json.dumps(feature_grad_line(args, dev)))
        return

    if args.kept_lattice:
        if rank == 0 and args.impl == "ours":
            print(json.dumps(kept_lattice_line(args, dev)))
        return

    if args.impl == "reference":
        if rank != 0:
            return
        fn, why = reference_impl()
        if fn is None:
            print(json.dumps({"impl": "reference", "unavailable": why}))
            return
        world_eff = 1
    else:
        fn = ours_impl()
        if args.lattice_precision != "fp32":
            from plattice_pytorch_b200 import PLOO
            PLOO.set_lattice_precision(args.lattice_precision)
        dist_init(world, local)
        world_eff = world

    if args.impl == "reference" and args.batch_split:   # the reference: the whole batch on one GPU
        imgs = load_inputs(args, 0, 1)
    else:
        imgs = load_inputs(args, rank, world_eff)
    h, w, pd = imgs[0]["features"].shape
    vd = imgs[0]["values"].shape[2]
    n = h * w
    n_images = len(imgs)
    batch = []
    for im in imgs:
        f = torch.from_numpy(im["features"]).to(dev)
        v = torch.from_numpy(im["values"]).to(dev).requires_grad_(True)
        g = torch.from_numpy(im["grad"]).to(dev)
        batch.append((f, v, g))
    per_image_fn, per_image_batch = fn, batch
    batched = (args.batched or args.batch_split > 0) and args.impl == "ours"
    if batched:   # one [B,H,W,...] triple, one library call per step
        from plattice_pytorch_b200 import PermutoLatticeBatchFunction
        fn = PermutoLatticeBatchFunction
        batch = [(torch.stack([b[0] for b in batch]), torch.stack([b[1].detach() for b in batch]).requires_grad_(True),
                  torch.stack([b[2] for b in batch]))]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    if args.mode == "device":
        for _ in range(args.warmup):
            for (f, v, g) in batch:
                step(fn, f, v, g)
        t = timed_device(fn, batch, args.steps, flush)
        if rank == 0:
            print(json.dumps({"mode": "device", "impl": args.impl, "workload": args.workload,
                              "ms_per_step": t / args.steps}))
        return

    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world_eff)))
    clocks = ClockSampler([torch.device("cuda", i) for i in range(max(1, local_world if world_eff > 1 else 1))])
    if local == 0:
        clocks.start()
    # soak: untimed steps until clocks settle under load
    t_end = time.perf_counter() + args.soak_seconds
    while time.perf_counter() < t_end:
        for (f, v, g) in batch:
            step(fn, f, v, g)
        torch.cuda.synchronize()
    for _ in range(args.warmup):
        flush.fill_(1.0)
        for (f, v, g) in batch:
            step(fn, f, v, g)
    torch.cuda.synchronize()
    barrier(world_eff)
    torch.cuda.synchronize()
    host_us = []
    graphs0 = graph_stats(args.impl)
    per_step = timed_device(fn, batch, args.steps, flush, host_us)
    graphs1 = graph_stats(args.impl)
    torch.cuda.synchronize()
    barrier(world_eff)
    # the median step when there are enough steps for it to mean something,
    # else the mean; the slowest rank sets the job's time either way
    t_step = statistics.median(per_step) if args.steps >= 50 else sum(per_step) / len(per_step)
    t_step = max_over_ranks(t_step, world_eff)
    t_dev = t_step * args.steps
    host_med = max_over_ranks(statistics.median(host_us), world_eff)

    # end to end from pinned host buffers
    host = [(torch.from_numpy(im["features"]).pin_memory(), torch.from_numpy(im["values"]).pin_memory(),
             torch.from_numpy(im["grad"]).pin_memory()) for im in imgs]
    if batched:
        host = [tuple(torch.stack([hh[k] for hh in host]).pin_memory() for k in range(3))]
    for _ in range(max(1, args.warmup // 2)):
        timed_e2e(fn, host, 1, dev)
    barrier(world_eff)
    t_e2e = timed_e2e(fn, host, args.steps, dev)
    barrier(world_eff)
    t_e2e = max_over_ranks(t_e2e, world_eff)
    clk = clocks.stop()

    imgs_job = args.batch_split if args.batch_split else world_eff * n_images
    px_total = imgs_job * n * args.steps
    value = px_total / (t_dev * 1e-3) / 1e6
    h2d = sum(int(x.numel()) * 4 for hh in host for x in hh)
    d2h = sum(int(hh[1].numel()) * 4 for hh in host)   # the value gradient
    res = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world_eff, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_dev / args.steps, "higher_is_better": True,
        "scaling": "strong" if args.batch_split else "weak", "vs_baseline": None,
        "timing": ("median" if args.steps >= 50 else "mean") + " of the K per-step CUDA-event times "
                  "(max over ranks)",
        "ms_per_step_mean": max_over_ranks(sum(per_step) / len(per_step), world_eff),
        "host_enqueue_us_per_step": host_med,
        "dtype": "f32" if args.lattice_precision == "fp32" or args.impl == "reference"
                 else "f32 (bf16 rows in the streaming blur passes)",
        "data": "synthetic",
        "config": {"workload": args.workload, "h": h, "w": w, "pd": pd, "vd": vd,
                   "images_per_gpu": n_images, "images_per_job": imgs_job,
                   "l2": "flushed between timed steps (256 MiB write, outside the events)",
                   "parallelism": (f"{imgs_job} images split by image over {world_eff} rank(s), no collective"
                                   if args.batch_split else
                                   "one image lattice per rank, no collective" if world_eff > 1 else "1 GPU"),
                   "api": ("PermutoLatticeBatchFunction (one call per batch)" if batched else
                           "PermutoLatticeFunction forward") + " + torch.autograd.grad backward"},
        "e2e": {"value": px_total / (t_e2e * 1e-3) / 1e6, "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "pipeline": "H2D of features, values and upstream gradient on an input stream, filter on "
                            "the default stream, D2H of the value gradient (the step's result) on an output "
                            "stream, ordered by events (identical for both arms)"},
        "clocks": clk,
    }
    if args.impl == "reference":
        res["impl"] = "reference"
        res["reference_build"] = "reference permuto.cpp + permutohedral.cu, unmodified, nvcc sm_100a"

    if args.impl == "ours":
        if batched:
            info, prof = profile_ours(fn, batch, args.profile_steps, flush, True)
            _, gprof = profile_ours(fn, batch, args.profile_steps, flush, True, groups=True)
            n_prof, launch_mult = n * n_images, 1   # the batch's pixels, one call per step
        else:
            info, prof = profile_ours(per_image_fn, per_image_batch, args.profile_steps, flush, False)
            _, gprof = profile_ours(per_image_fn, per_image_batch, args.profile_steps, flush, False, groups=True)
            n_prof, launch_mult = n, n_images
        n = n_prof
        m, u, cap = info["m"], info["u_total"], info["cap_log2"]
        peak, peak_kind = hbm_peak()
        per_stage = {}
        launches_per_step = 0
        for st, (ms, cnt) in prof.items():
            if cnt == 0 or st in ("build", "filter_fwd", "filter_bwd"):
                continue
            launches_per_step += cnt / args.profile_steps
            kb = kernel_bytes(st, n, pd, vd, m, u, cap)
            step_ms = ms / args.profile_steps
            per_stage[st] = {"ms_per_step": step_ms, "launches_per_step": cnt / args.profile_steps,
                             "avg_launch_us": ms / cnt * 1e3, "bytes_per_step": kb,
                             "gbs": kb / (step_ms * 1e-3) / 1e9}
        dom = max(per_stage, key=lambda k: per_stage[k]["ms_per_step"])
        d = per_stage[dom]
        ach = d["gbs"]
        res["roofline"] = {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": peak, "unit": "GB/s",
                           "frac": ach / peak, "peak_kind": peak_kind,
                           "traffic": traffic_from_profiles(dom),
                           "bytes_per_step": d["bytes_per_step"],
                           "launches_per_step": d["launches_per_step"]}
        b_fwd, b_bwd = stage_bytes(n, pd, vd, m)
        stage_ms = sum(per_stage[s]["ms_per_step"] for s in per_stage
                       if s in ("splat_fwd", "blur_fwd", "slice_fwd", "zero", "splat_bwd", "blur_bwd", "slice_bwd"))
        all_ms = sum(per_stage[s]["ms_per_step"] for s in per_stage)
        group_ms = (gprof.get("filter_fwd", (0.0, 0))[0] + gprof.get("filter_bwd", (0.0, 0))[0]) / args.profile_steps
        build_ms = gprof.get("build", (0.0, 0))[0] / args.profile_steps
        res["roofline_stages"] = {
            "definition": "(B_fwd + B_bwd) of splat+blur+slice / device time of the launches that do them: "
                          "the forward's launches after the lattice build (the splat launch also runs the "
                          "blur-neighbour lookups) and the backward's, timed with one event pair per group "
                          "(kernel_ms); kernel_ms_per_launch_events sums per-launch event intervals instead "
                          "(each holds 2-3 us of event overhead); B per the lattice byte formula",
            "bytes": b_fwd + b_bwd, "kernel_ms": group_ms, "build_ms": build_ms,
            "kernel_ms_per_launch_events": stage_ms,
            "achieved": (b_fwd + b_bwd) / (group_ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
            "frac": (b_fwd + b_bwd) / (group_ms * 1e-3) / 1e9 / peak,
            "frac_per_launch_events": (b_fwd + b_bwd) / (stage_ms * 1e-3) / 1e9 / peak,
            "frac_end_to_end": (b_fwd + b_bwd) / ((t_dev / args.steps) * 1e-3) / 1e9 / peak,
            "frac_all_kernels": (b_fwd + b_bwd) / (all_ms * 1e-3) / 1e9 / peak}
        res["stages"] = per_stage
        res["lattice"] = {"m": m, "u_total": u, "cap_log2": cap}
        K = pd + 1
        res["atomics"] = {
            "reference_scalar_atomics_fwd": n * K * (vd + 1),   # permutohedral.cu:316-318, one per slot and channel
            "reference_scalar_atomics_bwd": n * K * vd,
            "measured": atomics_from_profiles() if args.workload == "voronoi1024_pd5_vd3" else {},
            "measured_source": "profiles/atomics.txt (ncu, one launch each, this workload)"}
        res["gpu_launches"] = int(round(launches_per_step * args.steps * launch_mult))
        cap, rep = graph_stats(args.impl)
        res["call_graphs"] = {"captured": cap, "replayed": rep,
                              "captured_in_timed_steps": graphs1[0] - graphs0[0],
                              "replayed_in_timed_steps": graphs1[1] - graphs0[1],
                              "note": "calls repeated with the same buffers run as one CUDA graph launch"}

    if rank == 0 and world_eff == 1 and not args.no_cpu_baseline:
        im = imgs[0]
        res["cpu_baseline"] = cpu_baseline(im["features"], im["values"], im["grad"], args.cpu_sample)
        res["cpu_lattice_oracle"] = cpu_lattice_oracle(im["features"], im["values"], im["grad"])
    if rank == 0:
        print(json.dumps(res))
    if world_eff > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
