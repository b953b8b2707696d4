#!/usr/bin/env python
"""Headline benchmark: fwd+bwd soft-DTW DP cells/s, B=4096 pairs, N=M=1024, D=64, fp32.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = soft-DTW forward + backward (gradients for X and Y) over the whole
batch through the public API (torchwarp_b200.functional.soft_dtw, gamma=0.01,
squared-Euclidean cost).  With N GPUs (torchrun, one process per GPU) the
batch of 4096 pairs is sharded N ways (strong scaling); the only exchange is
an NCCL all_gather of the per-pair distances.

Printed (rank 0), one JSON line:
  value     cells/s over all GPUs, inputs resident in HBM, timed with CUDA
            events between barriers, max over ranks;
  e2e       the same step with X, Y copied from pinned host memory and the
            distances copied back inside the timed region;
  roofline  the dominant native kernel (longest average launch): its
            algorithmic bytes per launch / its average CUDA-event duration in
            the timed region, against MEASURED_PEAKS.json, with the DRAM
            traffic ncu measured for that kernel (per cell, scaled);
  cpu_baseline  the reference's own float32 PyTorch CPU backend on every host
            thread, on a bounded sample of the same workload (rank 0, N=1
            only); the float64 C port under oracle/ where the reference
            package is not present.
``--impl reference`` times that CPU implementation of the reference's path
on the same workload and prints the same line with "impl": "reference".
``--impl reference-cuda`` times the reference's own CUDA kernels (its
JIT-built extensions, float32) on the same inputs, in chunks of pairs, as a
secondary line with "impl": "reference-cuda".
The reference package is read from baseline/_ref (not part of this
package; the comparison arms only).
"""

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fwd+bwd DP cells/s (soft-DTW B=4096 N=M=1024)"
UNIT = "cells/s"
ALGO_BYTES_PER_CELL = 8      # soft-DTW fwd+bwd: cost read + cost-gradient write

# Per native call: (kernel launches per call, algorithmic bytes per cell of one
# launch, DRAM bytes per cell of one launch measured by ncu).  Algorithmic:
# the DP forward's cost read and the backward's cost-gradient write (the
# 8 B/cell of the step split between them), the cost builder's cost write,
# each chain-rule launch's cost-gradient read.  Measured: dram__bytes_read.sum
# + dram__bytes_write.sum of one launch of each kernel, captured one kernel at
# a time.  The DP sweeps and the chain rule were captured on the timed rows'
# shape (N=M=1024, D=64, gamma=0.01) at B=256, since what the backward and the
# chain rule skip depends on the rows, not the batch; the chain rule's figure
# less its own gradient write, which is added back at the timed shape.  The
# cost builder was captured at B=4096, N=M=256, less its X, Y read at that N
# (added back at the timed shape).
CALLS = {
    "udtw_cost": (1, 4, 3.91),           # C write + mask
    "sdtw_forward": (1, 4, 8.06),        # C read + saved R' write + edge stream
    "sdtw_backward": (1, 4, 0.79),       # the saved rows and the dC tiles (with the bit
                                         # mask) next to the alignment corridor, mask, edge
    "udtw_features_grad": (2, 4, 1.18),  # the chunks of dC the backward flagged nonzero, their
                                         # mask words and features (dense: 5.95)
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-cuda"])
    ap.add_argument("--chunk", type=int, default=512,
                    help="pairs per call of the reference's CUDA path (memory bound)")
    ap.add_argument("--batch", type=int, default=4096)
    ap.add_argument("--length", type=int, default=1024)
    ap.add_argument("--dim", type=int, default=64)
    ap.add_argument("--gamma", type=float, default=0.01)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--workload", default="cfg5",
                    choices=["cfg5", "cfg5-udtw", "cfg1", "cfg2", "cfg3", "cfg4", "cfg4-cost",
                             "train-ecg"],
                    help="cfg5 (default) is the headline line; the others time the remaining "
                         "configurations on one GPU (secondary lines, same JSON shape)")
    return ap.parse_args()


def config(a, world):
    return {"workload": "soft_dtw fwd+bwd, squared-Euclidean cost, gamma={}".format(a.gamma),
            "global_batch": a.batch, "N": a.length, "M": a.length, "D": a.dim,
            "per_gpu_batch": -(-a.batch // world), "parallelism": "dp{}".format(world),
            "l2": "inputs larger than L2 (X,Y {:.1f} GB, cost {:.1f} GB)".format(
                2 * a.batch // world * a.length * a.dim * 4 / 1e9,
                a.batch // world * a.length * a.length * 4 / 1e9)}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# --------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clock, power and clock-event reasons with NVML every 200 ms."""

    NAMES = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
             0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device):
        self.samples, self.stop, self.h, self.max_mhz = [], threading.Event(), None, None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.nv = pynvml
        except Exception:  # sampling is best effort; the number is still reported
            self.h = None

    def _run(self):
        nv = self.nv
        while not self.stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)))
            except Exception:
                pass
            self.stop.wait(0.2)

    def __enter__(self):
        if self.h is not None:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.h is not None:
            self.stop.set()
            self.t.join()
        return False

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        mhz = [s[0] for s in self.samples]
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = [n for bit, n in self.NAMES.items() if mask & bit]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz)}


# --------------------------------------------------------------- ours

def run_ours(a):
    import torch.distributed as dist

    import torchwarp_b200 as twb
    from torchwarp_b200 import _native

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    from torchwarp_b200.sharding import gather_pairs, shard_bounds
    lo, hi = shard_bounds(a.batch, world, rank)
    Bl, N, D = hi - lo, a.length, a.dim
    cells_total = a.batch * N * N
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    X = torch.randn(Bl, N, D, device=dev, generator=g)
    Y = torch.randn(Bl, N, D, device=dev, generator=g)

    def step(x, y):
        x = x.detach().requires_grad_(True)
        y = y.detach().requires_grad_(True)
        d = twb.functional.soft_dtw(x, y, gamma=a.gamma)
        d.sum().backward()
        if world > 1:
            gather_pairs(d.detach(), a.batch)   # every rank gets all B distances
        return d, x.grad, y.grad

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(fn, steps):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    for _ in range(a.warmup):
        step(X, Y)
    with ClockSampler(local) as clk, _native.LaunchTimer() as lt:
        ms = timed(lambda: step(X, Y), a.steps)
    torch.cuda.synchronize()
    kern = lt.totals()
    ms_step = ms / a.steps
    value = cells_total / (ms_step / 1e3)

    e2e = None
    if not a.no_e2e:
        # Host-resident inputs (pinned), copied to the device every step and
        # the distances read back every step.  The copy of step k+1 runs on a
        # copy stream while step k computes (double-buffered device inputs),
        # as a training loop with a prefetching loader would.
        Xh = X.cpu().pin_memory()
        Yh = Y.cpu().pin_memory()
        out_h = torch.empty(2, Bl, pin_memory=True)
        copy_stream = torch.cuda.Stream(dev)
        bufs = [(torch.empty_like(X), torch.empty_like(Y)) for _ in range(2)]
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]
        for e in free:
            e.record()

        def issue_copy(k):
            s = k % 2
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(free[s])
                bufs[s][0].copy_(Xh, non_blocking=True)
                bufs[s][1].copy_(Yh, non_blocking=True)
                ready[s].record(copy_stream)

        def e2e_run(steps):
            issue_copy(0)
            for k in range(steps):
                if k + 1 < steps:
                    issue_copy(k + 1)
                s = k % 2
                torch.cuda.current_stream().wait_event(ready[s])
                d, _, _ = step(bufs[s][0], bufs[s][1])
                out_h[s].copy_(d.detach(), non_blocking=True)
                free[s].record()

        # The first step's copy has nothing to overlap with (pipeline fill);
        # it stays inside the timed region, spread over at least 20 steps as
        # in a long training loop.
        e2e_steps = max(a.steps, 20)
        e2e_run(2)
        ms_e = timed(lambda: e2e_run(e2e_steps), 1)
        del bufs
        e2e = {"value": cells_total / (ms_e / e2e_steps / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int((Xh.numel() + Yh.numel()) * 4 * world),
               "d2h_bytes_per_step": int(Bl * 4 * world), "ms_per_step": ms_e / e2e_steps,
               "steps": e2e_steps,
               "copies": "pinned host -> device every step, overlapped with the previous "
                         "step on a copy stream; distances read back every step; the first "
                         "copy (pipeline fill) is inside the timed region"}

    # dominant native kernel of the timed region (one C-ABI call may launch
    # several kernels of equal work: the chain rule runs its dX and dY sides)
    def per_launch(kv):
        name, (calls, tot) = kv
        return tot / (calls * CALLS.get(name, (1, 0, 0))[0])

    name, (calls, tot) = max(kern.items(), key=per_launch)
    launches_per_call, algo_pc, traffic_pc = CALLS.get(name, (1, 0, None))
    per_launch_ms = tot / (calls * launches_per_call)
    peak, src = peaks()
    cells_local = Bl * N * N
    feat = Bl * N * D * 4                 # one side's features
    algo = cells_local * algo_pc
    traffic = None if traffic_pc is None else cells_local * traffic_pc
    if name == "udtw_cost":
        algo += 2 * feat
        traffic += 2 * feat
    elif name == "udtw_features_grad":
        algo += feat                      # each side writes its own gradient
        traffic += feat
    achieved = algo / (per_launch_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": peak,
                "unit": "GB/s", "frac": achieved / peak, "peak_source": src,
                "traffic": traffic,
                "traffic_source": "ncu dram__bytes_read+write per cell of one launch of this "
                                  "kernel, captured alone on the timed rows' shape at B=256 "
                                  "(N=M=1024, D=64), scaled to this launch's cells",
                "algorithmic_bytes_per_launch": algo, "avg_launch_ms": per_launch_ms,
                "launches_per_call": launches_per_call,
                "step_frac": (cells_local * ALGO_BYTES_PER_CELL / (ms_step / 1e3) / 1e9) / peak,
                "kernels_ms_per_step": {k: v[1] / a.steps for k, v in kern.items()}}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        cpu = cpu_baseline(a, X, Y)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    launches_per_step = sum(v[0] for v in kern.values()) // a.steps
    gpu_launches = sum(CALLS.get(k, (1,))[0] * v[0] for k, v in kern.items())
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config(a, world), "e2e": e2e, "roofline": roofline,
            "cpu_baseline": cpu, "clocks": clk.summary(), "gpu_launches": gpu_launches,
            "native_calls_per_step": launches_per_step}
    _emit(line)


# --------------------------------------------------------------- CPU arms

REF_DIR = ROOT / "baseline" / "_ref"


def _reference_package():
    """The reference package (hibana2077/torchwarp) from baseline/_ref, or None."""
    if not (REF_DIR / "torchwarp" / "__init__.py").exists():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    try:
        import torchwarp.functional as ref_F
    except Exception:  # pragma: no cover
        return None
    return ref_F


def _cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:  # pragma: no cover
        pass
    return "unknown CPU"


def _ref_cpu_step(ref_F, Xs, Ys, gamma):
    x = Xs.clone().requires_grad_(True)
    y = Ys.clone().requires_grad_(True)
    ref_F.soft_dtw(x, y, gamma=gamma, backend="torch").sum().backward()


def _ref_cpu_inputs(a, pairs):
    g = torch.Generator().manual_seed(1234)
    return (torch.randn(pairs, a.length, a.dim, generator=g),
            torch.randn(pairs, a.length, a.dim, generator=g))


def _oracle_sample(Xs, Ys, gamma):
    import oracle
    oracle.soft_dtw(Xs, Ys, gamma=gamma)


def cpu_baseline(a, X, Y, sample_pairs=16):
    """The reference's float32 PyTorch CPU backend on every host thread, on
    two pairs of the workload; without the reference package, the float64
    oracle on one thread on the first pairs of the same inputs."""
    ref_F = _reference_package()
    if ref_F is not None:
        threads = os.cpu_count() or 1
        prev = torch.get_num_threads()
        torch.set_num_threads(threads)
        try:
            Xs, Ys = _ref_cpu_inputs(a, 2)
            _ref_cpu_step(ref_F, Xs[:1, :64], Ys[:1, :64], a.gamma)   # warm-up
            t0 = time.perf_counter()
            _ref_cpu_step(ref_F, Xs, Ys, a.gamma)
            dt = time.perf_counter() - t0
        finally:
            torch.set_num_threads(prev)
        cells = 2 * a.length * a.length
        return {"value": cells / dt, "unit": UNIT, "cores": threads, "kind": "reference",
                "sample": "2 of the {} pairs (N=M={}, D={}), the reference's float32 PyTorch "
                          "CPU backend (backend='torch'), fwd+bwd, {} threads on {}, "
                          "{:.1f} s".format(a.batch, a.length, a.dim, threads, _cpu_model(), dt)}
    import oracle
    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover
        threadpool_limits = None
    oracle.lib()
    Xs = X[:sample_pairs].double().cpu().numpy()
    Ys = Y[:sample_pairs].double().cpu().numpy()
    ctx = threadpool_limits(1) if threadpool_limits else None
    t0 = time.perf_counter()
    if ctx:
        with ctx:
            _oracle_sample(Xs, Ys, a.gamma)
    else:
        _oracle_sample(Xs, Ys, a.gamma)
    dt = time.perf_counter() - t0
    cells = sample_pairs * a.length * a.length
    return {"value": cells / dt, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": "{} of the {} pairs (N=M={}, D={}), float64 fwd+bwd, {:.1f} s".format(
                sample_pairs, a.batch, a.length, a.dim, dt)}


def run_reference(a):
    """The reference's own CPU implementation of the path: its float32
    PyTorch backend (backend='torch') from baseline/_ref on every host thread,
    each step a chunk of pairs of the workload.  Without the reference
    package, its restatement in oracle/ (float64 C, all threads)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return
    threads = os.cpu_count() or 1
    ref_F = _reference_package()
    if ref_F is not None:
        torch.set_num_threads(threads)
        pairs = 2
        Xs, Ys = _ref_cpu_inputs(a, pairs)
        for _ in range(a.warmup):
            _ref_cpu_step(ref_F, Xs[:, :256], Ys[:, :256], a.gamma)
        t0 = time.perf_counter()
        for _ in range(a.steps):
            _ref_cpu_step(ref_F, Xs, Ys, a.gamma)
        dt = (time.perf_counter() - t0) / a.steps
        kind, dtype = "reference", "f32"
        sample = ("{} pairs per step (N=M={}, D={}) of the {}-pair workload, the reference's "
                  "float32 PyTorch CPU backend (backend='torch'), fwd+bwd, {} threads on {}; "
                  "warm-up steps on 256-step prefixes".format(pairs, a.length, a.dim, a.batch,
                                                               threads, _cpu_model()))
    else:
        from concurrent.futures import ThreadPoolExecutor

        import oracle
        try:
            from threadpoolctl import threadpool_limits
        except ImportError:  # pragma: no cover
            threadpool_limits = None
        oracle.lib()
        pairs = threads
        rng = np.random.default_rng(1234)
        Xn = rng.standard_normal((pairs, a.length, a.dim))
        Yn = rng.standard_normal((pairs, a.length, a.dim))

        def one(i):
            oracle.soft_dtw(Xn[i:i + 1], Yn[i:i + 1], gamma=a.gamma)

        def sample():
            with ThreadPoolExecutor(threads) as ex:
                list(ex.map(one, range(threads)))

        ctx = threadpool_limits(1) if threadpool_limits else None
        if ctx:
            ctx.__enter__()
        for _ in range(a.warmup):
            sample()
        t0 = time.perf_counter()
        for _ in range(a.steps):
            sample()
        dt = (time.perf_counter() - t0) / a.steps
        if ctx:
            ctx.__exit__(None, None, None)
        kind, dtype = "port", "f64"
        sample = ("{} pairs per step (N=M={}, D={}) of the {}-pair workload, the float64 C "
                  "restatement in oracle/ (no reference package present), {} threads".format(
                      pairs, a.length, a.dim, a.batch, threads))
    cells = pairs * a.length * a.length
    value = cells / dt
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
            "config": config(a, world), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    _emit(line)


def run_reference_cuda(a):
    """The reference's own CUDA kernels (JIT-built from baseline/_ref's
    csrc on this GPU, float32, backend='cuda'), on the same workload in
    chunks of --chunk pairs: one step is every chunk's fwd+bwd."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    ref_F = _reference_package()
    if ref_F is None:
        _emit({"impl": "reference-cuda", "unavailable": "reference package not in baseline/_ref"})
        return
    from torchwarp import _cuda as ref_cuda
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ext = "jeanie" if a.workload in ("cfg3", "cfg4") else "udtw"
    t_build = time.perf_counter()
    if ref_cuda.load(ext) is None:
        _emit({"impl": "reference-cuda",
               "unavailable": "its CUDA extension did not build: {}".format(
                   ref_cuda.build_error(ext))})
        return
    t_build = time.perf_counter() - t_build
    g = torch.Generator(device=dev).manual_seed(1234)
    metric, algo_per_step = METRIC, None
    if a.workload in ("cfg5", "cfg5-udtw"):
        X = torch.randn(a.batch, a.length, a.dim, device=dev, generator=g)
        Y = torch.randn(a.batch, a.length, a.dim, device=dev, generator=g)
        SX = torch.rand(a.batch, a.length, 1, device=dev, generator=g) + 0.5
        SY = torch.rand(a.batch, a.length, 1, device=dev, generator=g) + 0.5
        cells = a.batch * a.length * a.length
        batch = a.batch
        if a.workload == "cfg5-udtw":
            metric = "fwd+bwd DP cells/s (uDTW B={} N=M={} D={}, beta=1)".format(
                a.batch, a.length, a.dim)
            algo_per_step = 16 * cells

        def one(b0, b1):
            x = X[b0:b1].detach().requires_grad_(True)
            y = Y[b0:b1].detach().requires_grad_(True)
            if a.workload == "cfg5":
                ref_F.soft_dtw(x, y, gamma=a.gamma, backend="cuda").sum().backward()
            else:
                sx = SX[b0:b1].detach().requires_grad_(True)
                sy = SY[b0:b1].detach().requires_grad_(True)
                d, p = ref_F.udtw(x, y, sx, sy, gamma=a.gamma, beta=1.0, backend="cuda")
                (d + p).sum().backward()
    else:
        K = (15,) if a.workload == "cfg3" else (7, 7)
        batch = 1024
        Q = torch.randn(batch, *K, 10, 256, device=dev, generator=g)
        S = torch.randn(batch, 10, 256, device=dev, generator=g)
        cells = batch * int(np.prod(K)) * 100
        if a.workload == "cfg3":
            metric = "fwd+bwd DP cells/s (JEANIE B=1024 K=15 T=U=10 D=256)"
            algo_per_step = 335544320
        else:
            metric = "fwd+bwd DP cells/s (FVM B=1024 K1=K2=7 T=U=10 D=256)"
            algo_per_step = 1048576000

        def one(b0, b1):
            q = Q[b0:b1].detach().requires_grad_(True)
            s_ = S[b0:b1].detach().requires_grad_(True)
            if a.workload == "cfg3":
                ref_F.jeanie(q, s_, gamma=0.1, max_shift=1, backend="cuda").sum().backward()
            else:
                ref_F.fvm(q, s_, gamma=0.1, backend="cuda").sum().backward()
    chunk = min(a.chunk, batch)
    if algo_per_step is None:
        algo_per_step = ALGO_BYTES_PER_CELL * cells

    def step():
        for b0 in range(0, batch, chunk):
            one(b0, min(batch, b0 + chunk))

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    peak, src = peaks()
    achieved = algo_per_step / (ms / 1e3) / 1e9
    _emit({"metric": metric, "value": cells / (ms / 1e3), "unit": UNIT, "n_gpus": 1,
           "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
           "dtype": "f32", "data": "synthetic",
           "config": config(a, 1) if a.workload.startswith("cfg5") else {"workload": a.workload},
           "impl": "reference-cuda", "chunk_pairs": chunk, "jit_build_s": round(t_build, 1),
           "roofline": {"bound": "hbm", "kernel": "whole step",
                        "algorithmic_bytes_per_step": algo_per_step,
                        "achieved": achieved, "peak": peak, "unit": "GB/s",
                        "frac": achieved / peak, "peak_source": src}})


# ------------------------------------------------- secondary workloads

def _secondary(a):
    """One GPU, inputs resident, fwd+bwd per step, CUDA-event timed; the
    reference's other benchmark configurations (seeded synthetic inputs with
    their shapes), the uDTW variant of cfg5 and a training step.  Algorithmic
    bytes follow the byte accounting of each configuration."""
    import torchwarp_b200 as twb
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(4321)
    w = a.workload

    def rn(*shape):
        return torch.randn(*shape, device=dev, generator=g)

    extra = {}

    if w == "cfg5-udtw":
        B, N, D = a.batch, a.length, a.dim
        X, Y = rn(B, N, D), rn(B, N, D)
        sx = torch.rand(B, N, 1, device=dev, generator=g) + 0.5
        sy = torch.rand(B, N, 1, device=dev, generator=g) + 0.5
        cells, algo = B * N * N, 16 * B * N * N
        metric = "fwd+bwd DP cells/s (uDTW B={} N=M={} D={}, beta=1)".format(B, N, D)

        def step():
            x, y = X.detach().requires_grad_(True), Y.detach().requires_grad_(True)
            a_, b_ = sx.detach().requires_grad_(True), sy.detach().requires_grad_(True)
            out = twb.functional.udtw(x, y, a_, b_, gamma=a.gamma, beta=1.0)
            (out.distance + out.penalty).sum().backward()
    elif w == "cfg1":
        X, Y = rn(64, 30, 8), rn(64, 40, 8)
        sx = torch.rand(64, 30, 1, device=dev, generator=g) + 0.5
        sy = torch.rand(64, 40, 1, device=dev, generator=g) + 0.5
        cells, algo = 64 * 30 * 40, 16 * 64 * 30 * 40
        metric = "fwd+bwd DP cells/s (uDTW B=64 N=30 M=40 D=8)"

        def step():
            x, y = X.detach().requires_grad_(True), Y.detach().requires_grad_(True)
            a_, b_ = sx.detach().requires_grad_(True), sy.detach().requires_grad_(True)
            out = twb.functional.udtw(x, y, a_, b_, gamma=1.0, beta=1.0)
            (out.distance + out.penalty).mean().backward()
    elif w == "cfg2":
        def series():
            s_ = torch.cumsum(0.1 * rn(500, 140, 1), dim=1)
            return (s_ - s_.mean(1, keepdim=True)) / s_.std(1, keepdim=True)
        X, Y = series(), series()
        cells, algo = 500 * 140 * 140, 8 * 500 * 140 * 140
        metric = "fwd+bwd DP cells/s (soft-DTW B=500 N=M=140 D=1)"

        def step():
            x = X.detach().requires_grad_(True)
            twb.functional.soft_dtw(x, Y, gamma=0.1).sum().backward()
    elif w == "cfg3":
        Q, S_ = rn(1024, 15, 10, 256), rn(1024, 10, 256)
        cells, algo = 1024 * 15 * 10 * 10, 335544320
        metric = "fwd+bwd DP cells/s (JEANIE B=1024 K=15 T=U=10 D=256)"

        def step():
            q, s_ = Q.detach().requires_grad_(True), S_.detach().requires_grad_(True)
            twb.functional.jeanie(q, s_, gamma=0.1, max_shift=1).sum().backward()
    elif w == "cfg4":
        Q, S_ = rn(1024, 7, 7, 10, 256), rn(1024, 10, 256)
        cells, algo = 1024 * 49 * 10 * 10, 1048576000
        metric = "fwd+bwd DP cells/s (FVM B=1024 K1=K2=7 T=U=10 D=256)"

        def step():
            q, s_ = Q.detach().requires_grad_(True), S_.detach().requires_grad_(True)
            twb.functional.fvm(q, s_, gamma=0.1).sum().backward()
    elif w == "train-ecg":
        # One training step of a forecaster with the uDTW loss, in the shape
        # and settings of the reference's ECG5000 speed experiment
        # (experiments/ecg5000_speed.py:36-76, ecg5000_forecast.py config
        # "default"/"udtw"): 84 observed and 56 predicted samples, batch 50,
        # an MLP forecaster (84 -> 256 -> 56, ReLU), a sigma network
        # (56 -> 64 -> 56, sigma = 2 sigmoid + 0.1), uDTW gamma 0.1, beta 0.01,
        # Adam lr 1e-3.  ECG5000 is not available: the series are seeded
        # synthetic heartbeats (Gaussian waves plus noise, z-normalised).
        n_in, n_out, batch = 84, 56, 50
        t = torch.linspace(0.0, 1.0, n_in + n_out, device=dev)
        amp = torch.rand(500, 3, 1, device=dev, generator=g) + 0.5
        ctr = torch.rand(500, 3, 1, device=dev, generator=g)
        wid = 0.02 + 0.05 * torch.rand(500, 3, 1, device=dev, generator=g)
        beats = (amp * torch.exp(-0.5 * ((t - ctr) / wid) ** 2)).sum(1) + 0.05 * rn(500, 140)
        beats = (beats - beats.mean(1, keepdim=True)) / beats.std(1, keepdim=True)
        x_all, y_all = beats[:, :n_in], beats[:, n_in:]
        torch.manual_seed(42)
        f = torch.nn.Sequential(torch.nn.Linear(n_in, 256), torch.nn.ReLU(),
                                torch.nn.Linear(256, n_out)).to(dev)
        sig_net = torch.nn.Sequential(torch.nn.Linear(n_out, 64), torch.nn.ReLU(),
                                      torch.nn.Linear(64, n_out)).to(dev)

        def sigma(v):
            return 2.0 * torch.sigmoid(sig_net(v)) + 0.1

        crit = twb.UDTW(gamma=0.1, beta=0.01, normalize=False)
        opt = torch.optim.Adam(list(f.parameters()) + list(sig_net.parameters()), lr=1e-3,
                               capturable=True)
        cells, algo = batch * n_out * n_out, 16 * batch * n_out * n_out
        metric = "uDTW training steps (forecaster B=50, 84 -> 56 samples), DP cells/s"
        sx, sy = x_all.new_empty(batch, n_in), y_all.new_empty(batch, n_out)
        it = [0]

        def train_step():
            pred = f(sx)
            d, p_ = crit(pred.unsqueeze(-1), sy.unsqueeze(-1), sigma(pred).unsqueeze(-1),
                         sigma(sy).unsqueeze(-1))
            opt.zero_grad(set_to_none=False)
            (d + p_).mean().backward()
            opt.step()

        def next_batch():
            k = it[0]
            it[0] += 1
            idx = torch.arange(k * batch, (k + 1) * batch, device=dev) % x_all.shape[0]
            sx.copy_(x_all[idx])
            sy.copy_(y_all[idx])

        def eager_step():
            next_batch()
            train_step()

        # The step is launch-bound (about 30 small kernels), so it is captured
        # once as a CUDA graph: forecaster, sigma network, uDTW loss (native
        # cost, DP forward, DP backward, chain rule), backward and Adam.  The
        # graph is captured after warm-up steps on a side stream; every timed
        # step copies its batch into the captured inputs and replays.
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                eager_step()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            train_step()

        def step():
            next_batch()
            graph.replay()

        for _ in range(3):
            eager_step()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(a.steps):
            eager_step()
        t1.record()
        torch.cuda.synchronize()
        extra["eager_ms_per_step"] = t0.elapsed_time(t1) / a.steps
        extra["step"] = ("one CUDA-graph replay of forward, uDTW loss, backward and Adam, "
                         "after a copy of the batch into the captured inputs")
    else:  # cfg4-cost
        Cc = rn(1024, 7, 7, 10, 10).abs()
        cells, algo = 1024 * 49 * 10 * 10, 40140800
        metric = "fwd+bwd DP cells/s (fvm_from_cost B=1024 K1=K2=7 T=U=10)"

        def step():
            c = Cc.detach().requires_grad_(True)
            twb.functional.fvm_from_cost(c, gamma=0.1).sum().backward()

    from torchwarp_b200 import _native
    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    with _native.LaunchTimer() as lt:   # per native call, in a separate untimed pass
        step()
    torch.cuda.synchronize()
    calls = {k: round(v[1], 4) for k, v in lt.totals().items()}
    peak, src = peaks()
    achieved = algo / (ms / 1e3) / 1e9
    _emit({"metric": metric, "value": cells / (ms / 1e3), "unit": UNIT, "n_gpus": 1,
           "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
           "higher_is_better": True, "dtype": "f32", "data": "synthetic",
           "config": {"workload": w},
           "roofline": {"bound": "hbm", "kernel": "whole step",
                        "algorithmic_bytes_per_step": algo, "achieved": achieved,
                        "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                        "peak_source": src},
           "native_calls_ms": calls, **extra})


_JSON_FD = None


def _stdout_to_stderr():
    """Point file descriptor 1 at stderr for the whole run, so that whatever a
    library writes to stdout (NCCL's version banner, for one) lands on stderr,
    and keep a duplicate of the original stdout for the single JSON line."""
    global _JSON_FD
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)


def _emit(obj):
    """Write the result line, and nothing else, to the original stdout."""
    data = (json.dumps(obj) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
        return
    os.write(_JSON_FD, data)


def main():
    a = parse()
    _stdout_to_stderr()
    if a.impl == "reference":
        run_reference(a)
    elif a.impl == "reference-cuda":
        run_reference_cuda(a)
    elif a.workload != "cfg5":
        _secondary(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
