#!/usr/bin/env python
"""Soft-DTW forward+backward DP-cell throughput on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4a|c4b|c5]

Workloads (synthetic, seeded data with the configs' shapes and
value distributions):
  c2   B=32/GPU, N=M=512, D=64, x,y ~ N(0,1), gamma=1 (default; headline).  One
       step = SoftDTW(fused=...)(x, y).mean().backward() -> dL/dx, dL/dy.  The
       headline `value` is the default CUDA path (fused=None -> fused); the
       unfused path is reported under "modes".
  c3   B=16/GPU, N=M=4096, D=8, gamma=0.1, fused: x = phase-shifted sines + noise,
       y = x time-warped by a random monotone cubic map + noise.
  c4a  B=64/GPU, N=1024, M=768, D=128, N(0,1), gamma=1, unfused (headline), fused
       under "modes".
  c4b  B=64/GPU, N=M=1024, D=128, normalize=True (3B problems, cells = 3*B*N*M).
  c5   barycenter of 4096 sequences (length 100, D=3, random-phase sines with
       random shifts + noise), gamma=1, Adam lr 0.1; one step = one Adam
       iteration over the whole set, cells = 4096*100*100.  The set is sharded
       over the ranks (strong scaling; per step the sum over ranks of [gradient |
       loss] through peer memory, fused with the Adam step); the other
       workloads run B problems per rank (weak scaling, no collective).
The default run (c2) also times c3 and c5 and reports them under "workloads"
(their own ms per step, kernel breakdown, MUFU fraction and latency floor; for
c5 on several GPUs the NCCL all-reduce of the gradient buffer and the
peer-memory exchange + Adam kernel, each timed on its own).
Metric: DP cells per second summed over all GPUs.  `--impl reference` times the
reference's CPU algorithm (the oracle restatement in oracle/, all host
threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "sdtw-cuda-torch_b200"))

# name: (B, N, M, D, gamma, normalize, headline mode, other modes, description)
WORKLOADS = {
    "c2": (32, 512, 512, 64, 1.0, False, "fused", ("unfused",),
           "BASELINE config 2: B=32/GPU, N=M=512, D=64, gamma=1, fwd+bwd, mean reduction"),
    "c3": (16, 4096, 4096, 8, 0.1, False, "fused", (),
           "BASELINE config 3: B=16/GPU, N=M=4096, D=8, gamma=0.1, sines + time warp, fused fwd+bwd"),
    "c4a": (64, 1024, 768, 128, 1.0, False, "unfused", ("fused",),
            "BASELINE config 4a: B=64/GPU, N=1024, M=768, D=128, gamma=1, unfused fwd+bwd"),
    "c4b": (64, 1024, 1024, 128, 1.0, True, "fused", ("unfused",),
            "BASELINE config 4b: B=64/GPU, N=M=1024, D=128, normalize=True (3B problems), fwd+bwd"),
    "c5": (4096, 100, 100, 3, 1.0, False, "barycenter", (),
           "BASELINE config 5: barycenter of 4096 sequences x 100 x 3, gamma=1, Adam lr=0.1, "
           "one step = one iteration over the whole set, sharded over the ranks"),
}
PUBLISHED = {  # the reference's published numbers: B=32 N=M=512 D=64 fwd+bwd (unstated GPU)
    "c2": {"fused": 32 * 512 * 512 / 0.14136, "unfused": 32 * 512 * 512 / 0.02010},
}
MUFU_PER_CELL = 7          # algorithmic ex2/lg2 per DP cell, forward + backward (reference algorithm)
MUFU_PER_SM_CLK = 16       # ex2/lg2 results per SM per clock
DEP_CYCLES = 49            # dependent chain of one exponential-domain step (SHFL, integer max/add-max/add,
                           # 2 FADD, FMUL), clock64 microbenchmark, one warp per SM sub-partition
# Algorithmic HBM bytes per DP cell of each library kernel: every table entry
# read or written once (cost 4 B, score 8 B as a (hi, lo) pair, E 4 B).
ALG_BYTES = {"cost_wl": 4, "cost_tc": 4, "wavefront_fwd": 12, "wavefront_bwd": 12, "wl_to_rm": 8, "grad_xy": 8,
             "rm_to_wl": 8, "cost_rowmajor": 4}
# Algorithmic MUFU ops per cell of the reference algorithm: forward softmin
# (2 ex2 + 1 lg2), reverse log-sum-exp (2 ex2 + 1 lg2) and E = exp(log E) (1 ex2).
ALG_MUFU = {"wavefront_fwd": 3, "wavefront_bwd": 4}
# DRAM bytes per launch measured by ncu (dram__bytes_read.sum + dram__bytes_write.sum,
# one launch each, cold L2) for the C2 workload, fused mode (profiles/c2_kernels_full.md).
TRAFFIC_C2 = {"wavefront_fwd": 55.90e6, "wavefront_bwd": 82.36e6, "cost_wl": 8.48e6, "grad_xy": 54.63e6}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    # Profiling runs: only the headline timed steps (no other modes, no end-to-end leg).
    ap.add_argument("--fused-only", action="store_true")
    # Profiling runs of one mode (it becomes the headline; implies --fused-only).
    ap.add_argument("--only-mode", default=None)
    # Profiling runs under a forced launch geometry: stripes per CTA x cluster size ("8x8").
    ap.add_argument("--plan", default=None)
    args = ap.parse_args()
    if args.only_mode:
        args.fused_only = True
    return args


# ----------------------------------------------------------------------------- data
def make_data(name, B, N, M, D, seed):
    """Seeded synthetic inputs with the shapes and value distributions of the
    BASELINE config (numpy float32)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    if name == "c3":
        t = np.arange(N, dtype=np.float64)
        f = rng.uniform(1, 8, size=(B, 1, D))
        ph = rng.uniform(0, 2 * np.pi, size=(B, 1, D))
        clean = np.sin(2 * np.pi * f * t[None, :, None] / N + ph)
        x = clean + 0.1 * rng.standard_normal((B, N, D))
        # y: x warped by w(u) = u + a u (1 - u)(1 - 2u), |a| < 0.8 (w' > 0, w(0) = 0, w(1) = 1).
        u = np.linspace(0.0, 1.0, M)
        a = rng.uniform(-0.8, 0.8, size=(B, 1))
        w = (u[None, :] + a * u[None, :] * (1 - u[None, :]) * (1 - 2 * u[None, :])) * (N - 1)
        y = np.empty((B, M, D))
        for bi in range(B):
            for c in range(D):
                y[bi, :, c] = np.interp(w[bi], t, clean[bi, :, c])
        y += 0.1 * rng.standard_normal((B, M, D))
        return x.astype(np.float32), y.astype(np.float32)
    if name == "c5":
        t = np.arange(N, dtype=np.float64)
        ph = rng.uniform(0, 2 * np.pi, size=(B, 1, D))
        k = np.arange(1, D + 1, dtype=np.float64)[None, None, :]
        shift = rng.integers(-10, 11, size=(B, 1, 1))
        ts = np.clip(t[None, :, None] - shift, 0, N - 1)  # edge-padded shift
        X = np.sin(2 * np.pi * ts / N * k + ph) + 0.2 * rng.standard_normal((B, N, D))
        return X.astype(np.float32), None
    x = rng.standard_normal((B, N, D)).astype(np.float32)
    y = rng.standard_normal((B, M, D)).astype(np.float32)
    return x, y


def cells_of(name):
    B, N, M, D, gamma, normalize, *_ = WORKLOADS[name]
    return (3 if normalize else 1) * B * N * M


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._th = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.max_mhz = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self._stop.clear()
            self._th = threading.Thread(target=self._run, daemon=True)
            self._th.start()
        return self

    def __exit__(self, *a):
        if self._th is not None:
            self._stop.set()
            self._th.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        nv = self._nv
        names = {
            "gpu_idle": getattr(nv, "nvmlClocksEventReasonGpuIdle", 0x1),
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        active = set()
        for _, r in self.samples:
            for k, bit in names.items():
                if k != "gpu_idle" and r & bit:
                    active.add(k)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(active), "samples": len(self.samples)}


# ----------------------------------------------------------------------------- CPU (oracle) timing
def time_oracle(name, budget_s):
    """Reference CPU algorithm (oracle/, all host threads) on a bounded sample
    of the workload: returns (cells/s, threads, sample description)."""
    import numpy as np
    from oracle import oracle as O

    B, N, M, D, gamma, normalize, mode, _, _ = WORKLOADS[name]
    if name == "c5":
        X, _ = make_data(name, B, N, M, D, seed=1234)
        sub = 256  # sequences per sampled iteration
        bary = X[:sub].mean(axis=0)
        x = np.broadcast_to(bary, (sub, N, D)).copy()
        y = X[:sub]
        kw = dict(gamma=gamma, grad_out=np.full(sub, 1.0 / B))
        unit_cells = sub * N * N
        desc = f"{sub} of 4096 sequences per iteration (loss and barycenter gradient)"
    else:
        per = N * M * (3 if normalize else 1)
        b_s = max(1, min(B, int(2e7 // per)))  # about one second of CPU work per call
        x, y = make_data(name, b_s, N, M, D, seed=1234)
        kw = dict(gamma=gamma, normalize=normalize, grad_out=np.full(b_s, 1.0 / B))
        unit_cells = (3 if normalize else 1) * b_s * N * M
        desc = (f"{b_s} of {B} problems ({N}x{M}, D={D}{', normalize' if normalize else ''}) per call, "
                "unfused reference algorithm")
    # Every host core, also under torchrun (which sets OMP_NUM_THREADS=1).
    O.set_num_threads(len(os.sched_getaffinity(0)))
    O.loss_and_grads(x, y, **kw)  # warm
    reps, t0 = 0, time.perf_counter()
    while reps == 0 or (time.perf_counter() - t0 < budget_s and reps < 1000):
        O.loss_and_grads(x, y, **kw)
        reps += 1
    dt = time.perf_counter() - t0
    return reps * unit_cells / dt, O.num_threads(), f"{reps} x {desc}, {dt:.1f} s"


def run_reference(args):
    name = args.workload
    B, N, M, D, gamma, normalize, mode, _, desc = WORKLOADS[name]
    cells = cells_of(name) if name != "c5" else B * N * N
    # Every step is a bounded sample (about two seconds) of the workload.
    for _ in range(max(args.warmup, 0)):
        time_oracle(name, 0.0)
    per_step, cores, sample = [], None, ""
    for _ in range(args.steps):
        v, cores, sample = time_oracle(name, 2.0)
        per_step.append(v)
    value = statistics.mean(per_step)
    line = {
        "impl": "reference", "metric": "fwd+bwd DP cells/s", "value": value, "unit": "cells/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * cells / value,
        "higher_is_better": True, "scaling": "strong" if name == "c5" else "weak", "vs_baseline": None,
        "dtype": "f32 (f64 DP)", "data": "synthetic, seeded (BASELINE config shapes and distributions)",
        "config": {"workload": f"{name}: {desc} (CPU: unfused; the reference has no CPU fused mode)",
                   "global_batch": B, "seq_len": N, "dim": D, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "cells/s", "cores": cores, "kind": "port",
                         "sample": sample + "; oracle/ restatement of launcher.py:305-368 + numpy cost and chain rule"},
        "e2e": {"value": value, "unit": "cells/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- our arm
def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            run_reference(args)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from softdtw_cuda import SoftDTW, _native
    from softdtw_cuda.distributed import shard_bounds, sharded_barycenter
    import softdtw_cuda.barycenters as _bc
    import softdtw_cuda.distributed as _dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def run_one(name, steps, warmup, fused_only, only_mode, sampler):
        """Times one workload; returns its measurements (all ranks)."""
        args_steps, args_warmup = steps, warmup
        B, N, M, Dm, gamma, normalize, head_mode, other_modes, desc = WORKLOADS[name]
        if only_mode:
            if only_mode not in (head_mode,) + tuple(other_modes):
                raise SystemExit(f"workload {name} has no mode {only_mode}")
            head_mode, other_modes = only_mode, ()
        is_bary = name == "c5"
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > 126 MB L2
        stream = torch.cuda.current_stream(dev)

        if is_bary:
            Xn, _ = make_data(name, B, N, M, Dm, seed=1234)
            lo, hi = shard_bounds(B, rank, world)
            X_h = torch.from_numpy(Xn[lo:hi]).pin_memory()
            X_d = X_h.to(dev)
            cells = B * N * N  # whole job per iteration
            my_cells = (hi - lo) * N * N
        else:
            xn, yn = make_data(name, B, N, M, Dm, seed=1234 + rank)
            x_h = torch.from_numpy(xn).pin_memory()
            y_h = torch.from_numpy(yn).pin_memory()
            x = x_h.to(dev)
            y = y_h.to(dev)
            cells = world * cells_of(name)
            my_cells = cells_of(name)

        # One loss module per mode, built once as a training loop does.
        loss_fn = {m: SoftDTW(gamma=gamma, normalize=normalize, fused=(None if m == "fused" else False))
                   for m in ("fused", "unfused")}

        def step(mode):
            xr = x.detach().requires_grad_(True)
            yr = y.detach().requires_grad_(True)
            out = loss_fn[mode](xr, yr)
            out.mean().backward()
            return xr.grad, yr.grad

        def timed(fn, k):
            times = []
            # About 0.7 ms of device work ahead of the first step (outside the
            # events): the first step then finds its kernels queued, as every
            # later step does, instead of the device waiting on the host's
            # first launches.
            for _ in range(16):
                flush.zero_()
            for _ in range(k):
                flush.zero_()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                times.append((e0, e1))
            torch.cuda.synchronize(dev)
            return [a.elapsed_time(b) for a, b in times]

        sampler = ClockSampler(local)
        modes = {}
        launches = 0
        breakdown = {}
        per_launch = {}
        all_modes = (head_mode,) + (() if fused_only else tuple(other_modes))
        with sampler:
            for mode in all_modes:
                allreduce_ms = None
                if is_bary:
                    # Kernel breakdown and launch count from one step-by-step
                    # call (per-kernel CUDA events cannot run inside a graph);
                    # a graph replay launches the same kernels.
                    _bc.USE_CUDA_GRAPH = False
                    sharded_barycenter(X_d, gamma=gamma, max_iter=args_warmup, lr=0.1, early_stopping=False)
                    torch.cuda.synchronize(dev)
                    barrier()
                    l0 = _native.launches()
                    _native.timing_enable(True)
                    sharded_barycenter(X_d, gamma=gamma, max_iter=args_steps, lr=0.1, early_stopping=False)
                    torch.cuda.synchronize(dev)
                    n_launch = _native.launches() - l0
                    kt = _native.timing_read()
                    _native.timing_enable(False)
                    _bc.USE_CUDA_GRAPH = True
                    # The all-reduce of [gradient | loss] on its own, as the
                    # iteration issues it.
                    allreduce_ms = 0.0
                    exchange_ms = None
                    if world > 1:
                        buf = torch.zeros(N * Dm + 1, device=dev)
                        for _ in range(5):
                            dist.all_reduce(buf)
                        torch.cuda.synchronize(dev)
                        barrier()
                        allreduce_ms = statistics.median(timed(lambda: dist.all_reduce(buf), 20))
                        ex = None
                        if _dist.USE_PEER_EXCHANGE:
                            try:
                                ex = _dist._PeerExchange(N * Dm, None, dev)
                            except (RuntimeError, ImportError, AttributeError) as err:
                                print(f"bench: no peer-memory exchange ({err})", file=sys.stderr)
                        if ex is not None:
                            # What the iteration runs instead: the peer-memory
                            # sum over ranks fused with the Adam step (one
                            # kernel), timed on scratch state.
                            kx = 30
                            st = dict(bary=torch.zeros(N, Dm, device=dev), m=torch.zeros(N, Dm, device=dev),
                                      v=torch.zeros(N, Dm, device=dev), lr=torch.full((kx,), 0.1, device=dev),
                                      step=torch.zeros(1, dtype=torch.int32, device=dev),
                                      lh=torch.zeros(kx, device=dev), bh=torch.zeros(kx, N, Dm, device=dev))

                            def sync_step():
                                _native.barycenter_sync_adam(buf, ex.peers, ex.world, ex.rank, ex.epoch, st["bary"],
                                                             st["m"], st["v"], st["lr"], st["step"], st["lh"],
                                                             st["bh"])

                            for _ in range(5):
                                sync_step()
                            torch.cuda.synchronize(dev)
                            barrier()
                            exchange_ms = statistics.median(timed(sync_step, 20))
                            torch.cuda.synchronize(dev)
                            barrier()
                            del ex
                    # The timed call: K iterations of the replayed CUDA graph
                    # (the untimed call of the same length captures it); the
                    # per-step figure is the average.
                    sharded_barycenter(X_d, gamma=gamma, max_iter=args_steps, lr=0.1, early_stopping=False)
                    torch.cuda.synchronize(dev)
                    barrier()
                    torch.cuda.synchronize(dev)
                    stats = {}
                    flush.zero_()
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    sharded_barycenter(X_d, gamma=gamma, max_iter=args_steps, lr=0.1, early_stopping=False, stats=stats)
                    e1.record(stream)
                    torch.cuda.synchronize(dev)
                    if not stats.get("graph") or stats.get("captured"):
                        raise SystemExit(f"barycenter timing did not replay a cached graph: {stats}")
                    ms = [e0.elapsed_time(e1) / args_steps] * args_steps
                else:
                    for _ in range(args_warmup):
                        step(mode)
                    torch.cuda.synchronize(dev)
                    barrier()
                    torch.cuda.synchronize(dev)
                    # The step time from K uninstrumented steps; then the same K
                    # steps again with per-kernel CUDA events on the launching
                    # stream (the kernel breakdown and the roofline's launch
                    # durations), whose event records would otherwise sit
                    # between the step's kernels.
                    l0 = _native.launches()
                    ms = timed(lambda: step(mode), args_steps)
                    n_launch = _native.launches() - l0
                    _native.timing_enable(True)
                    timed(lambda: step(mode), args_steps)
                    kt = _native.timing_read()
                    _native.timing_enable(False)
                bd = {k: v[0] / args_steps for k, v in kt.items()}
                pl = {k: v[0] / max(v[1], 1) for k, v in kt.items()}
                if mode == head_mode:
                    breakdown, per_launch, launches = bd, pl, n_launch
                torch.cuda.synchronize(dev)
                barrier()
                _native.check_status(dev)
                mean_ms = max_over_ranks(statistics.mean(ms))
                modes[mode] = {"value": cells / (mean_ms / 1e3), "ms_per_step": mean_ms,
                               "median_ms": statistics.median(ms), "kernel_ms_per_step": bd, "gpu_launches": n_launch}
                if allreduce_ms is not None:
                    # NCCL all-reduce of [grad | loss] on its own; the replayed
                    # iteration uses the peer-memory exchange when it is on.
                    modes[mode]["allreduce_ms_per_step"] = max_over_ranks(allreduce_ms)
                    if is_bary and world > 1:
                        modes[mode]["exchange_adam_ms_per_step"] = (max_over_ranks(exchange_ms)
                                                                    if exchange_ms is not None else None)
                pub = PUBLISHED.get(name, {}).get(mode)
                modes[mode]["vs_published"] = (modes[mode]["value"] / world / pub) if pub else None

        # End to end through the public API with host buffers.
        e2e = None
        if not fused_only:
            if is_bary:
                out_h = torch.empty(N, Dm).pin_memory()
                Xd = torch.empty_like(X_d)  # the device buffer the sequences are loaded into

                def e2e_run(k):
                    Xd.copy_(X_h, non_blocking=True)
                    bary = sharded_barycenter(Xd, gamma=gamma, max_iter=k, lr=0.1, early_stopping=False)
                    out_h.copy_(bary, non_blocking=True)

                e2e_run(args_steps)  # captures the graph the timed call replays
                torch.cuda.synchronize(dev)
                barrier()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                e2e_run(args_steps)
                e1.record(stream)
                torch.cuda.synchronize(dev)
                e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args_steps)
                h2d = X_h.numel() * 4 / args_steps
                d2h = out_h.numel() * 4 / args_steps
                api = ("softdtw_cuda.distributed.sharded_barycenter (pinned host sequences in, barycenter out; "
                       "per-step bytes = one call's copies / steps)")
            else:
                gx_h = torch.empty_like(x_h).pin_memory()
                gy_h = torch.empty_like(y_h).pin_memory()
                loss_h = torch.empty((), dtype=torch.float32).pin_memory()

                def e2e_step(grads_out):
                    xd = x_h.to(dev, non_blocking=True).requires_grad_(True)
                    yd = y_h.to(dev, non_blocking=True).requires_grad_(True)
                    loss = loss_fn[head_mode](xd, yd).mean()
                    loss.backward()
                    loss_h.copy_(loss.detach(), non_blocking=True)
                    if grads_out:
                        gx_h.copy_(xd.grad, non_blocking=True)
                        gy_h.copy_(yd.grad, non_blocking=True)

                # Headline: a training step's result (the loss) comes back to the
                # host; dL/dx, dL/dy are computed in the timed region and stay on
                # the device for the optimizer.  Also timed: the same step with both
                # gradients copied to host memory as well.
                res = {}
                for grads_out in (False, True):
                    for _ in range(args_warmup):
                        e2e_step(grads_out)
                    torch.cuda.synchronize(dev)
                    barrier()
                    res[grads_out] = max_over_ranks(statistics.mean(timed(lambda: e2e_step(grads_out), args_steps)))
                e2e_ms = res[False]
                h2d = x_h.numel() * 4 + y_h.numel() * 4
                d2h = 4
                d2h_grads = 4 + gx_h.numel() * 4 + gy_h.numel() * 4
                api = (f"softdtw_cuda.SoftDTW ({head_mode}; pinned host x,y in; loss out, dL/dx and dL/dy computed "
                       "and left on the device)")
                e2e_grads = {"value": cells / (res[True] / 1e3), "ms_per_step": res[True], "d2h_bytes_per_step": d2h_grads,
                             "api": f"as above, plus dL/dx and dL/dy copied to pinned host memory"}

                # The same K steps as one pipelined run, as a training loop
                # prefetches: step i+1's x, y copied on a copy stream into the
                # other of two device buffers while step i computes (the copy
                # engine runs beside the kernels); every step still copies its
                # inputs in and its loss out inside the timed region.  No L2
                # flush between steps (it would have to sit inside the region);
                # the inputs are fresh host copies every step.
                copy_st = torch.cuda.Stream(dev)
                bufs = [(torch.empty_like(x), torch.empty_like(y)) for _ in range(2)]
                copied = [torch.cuda.Event() for _ in range(2)]
                consumed = [torch.cuda.Event() for _ in range(2)]
                loss_hs = torch.empty(max(args_steps, args_warmup), dtype=torch.float32).pin_memory()

                def pipelined(k):
                    with torch.cuda.stream(copy_st):
                        copy_st.wait_stream(stream)
                        bufs[0][0].copy_(x_h, non_blocking=True)
                        bufs[0][1].copy_(y_h, non_blocking=True)
                        copied[0].record(copy_st)
                    for i in range(k):
                        cur = i % 2
                        if i + 1 < k:
                            nxt = (i + 1) % 2
                            with torch.cuda.stream(copy_st):
                                if i >= 1:
                                    copy_st.wait_event(consumed[nxt])
                                bufs[nxt][0].copy_(x_h, non_blocking=True)
                                bufs[nxt][1].copy_(y_h, non_blocking=True)
                                copied[nxt].record(copy_st)
                        stream.wait_event(copied[cur])
                        xd = bufs[cur][0].detach().requires_grad_(True)
                        yd = bufs[cur][1].detach().requires_grad_(True)
                        loss = loss_fn[head_mode](xd, yd).mean()
                        loss.backward()
                        loss_hs[i].copy_(loss.detach(), non_blocking=True)
                        consumed[cur].record(stream)

                pipelined(args_warmup)
                torch.cuda.synchronize(dev)
                barrier()
                flush.zero_()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                pipelined(args_steps)
                e1.record(stream)
                torch.cuda.synchronize(dev)
                pipe_ms = max_over_ranks(e0.elapsed_time(e1) / args_steps)
                e2e_pipe = {"value": cells / (pipe_ms / 1e3), "ms_per_step": pipe_ms, "h2d_bytes_per_step": h2d,
                            "d2h_bytes_per_step": d2h,
                            "api": "as the headline e2e, K steps in one run with the next step's host copies "
                                   "overlapped (copy stream, two device buffers); no L2 flush between steps"}
            e2e = {"value": cells / (e2e_ms / 1e3), "unit": "cells/s", "ms_per_step": e2e_ms,
                   "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "api": api}
            if not is_bary:
                e2e["grads_to_host"] = e2e_grads
                e2e["pipelined"] = e2e_pipe

        clocks = sampler.summary()
        head = modes[head_mode]

        # Roofline of the dominant kernel (largest device time per step).
        dom = max(breakdown, key=breakdown.get)
        dom_ms = per_launch[dom]
        launches_per_step = breakdown[dom] / dom_ms
        alg_bytes = ALG_BYTES.get(dom, 0) * my_cells / launches_per_step  # per launch
        peaks = {}
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                peaks = json.load(f)
        except OSError:
            pass
        hbm_peak = peaks.get("hbm_gbs", 6650.0)
        achieved = alg_bytes / (dom_ms / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                    "frac": achieved / hbm_peak,
                    "traffic": TRAFFIC_C2.get(dom) if name == "c2" else None,
                    "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                    "alg_bytes_per_cell": ALG_BYTES.get(dom, 0)}
        n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
        sm_mhz = clocks.get("sm_mhz") or peaks.get("sm_max_mhz", 1965.0)
        mufu_peak = n_sm * MUFU_PER_SM_CLK * sm_mhz * 1e6
        step_mufu = MUFU_PER_CELL * my_cells / (head["ms_per_step"] / 1e3)
        wf = {k: ALG_MUFU[k] * my_cells / (breakdown[k] / 1e3) for k in ALG_MUFU if k in breakdown}
        roofline_mufu = {"bound": "mufu", "unit": "Gop/s", "peak": mufu_peak / 1e9,
                         "peak_basis": f"{n_sm} SMs x {MUFU_PER_SM_CLK} ex2/lg2 per clk x {sm_mhz:.0f} MHz (median under load)",
                         "step_achieved": step_mufu / 1e9, "step_frac": step_mufu / mufu_peak,
                         "kernels": {k: {"achieved": v / 1e9, "frac": v / mufu_peak, "ms_per_step": breakdown[k],
                                         "alg_ops_per_cell": ALG_MUFU[k]} for k, v in wf.items()},
                         "alg_ops_per_cell": MUFU_PER_CELL}
        # Latency floor of the wavefronts: a problem needs N + M - 1 dependent
        # anti-diagonal steps (n_bands * (M + 32) when its stripes loop over bands),
        # each at least one cell's dependency chain (DEP_CYCLES, measured with
        # clock64 microbenchmarks on B200); problems beyond what fits at once run
        # in further waves.
        n_prob = (hi - lo) if is_bary else (3 if normalize else 1) * B
        Mp = N if is_bary else M
        pinfo = _native.plan_info(n_prob, N, Mp)
        steps = max(N + Mp - 1, pinfo["bands"] * (Mp + 32))
        waves = -(-n_prob // max(1, pinfo["clusters_fit"]))
        floor_ms = waves * steps * DEP_CYCLES / (sm_mhz * 1e6) * 1e3
        roofline_latency = {"bound": "dependent chain", "unit": "ms", "cycles_per_step": DEP_CYCLES,
                            "steps": steps, "waves": waves, "floor_ms": floor_ms,
                            "kernels": {k: {"ms_per_step": breakdown[k], "frac": floor_ms / breakdown[k]}
                                        for k in ALG_MUFU if k in breakdown}}


        return {"name": name, "B": B, "N": N, "M": M, "Dm": Dm, "desc": desc, "head_mode": head_mode,
                "is_bary": is_bary, "cells": cells, "modes": modes, "breakdown": breakdown, "launches": launches,
                "e2e": e2e, "roofline": roofline, "roofline_mufu": roofline_mufu,
                "roofline_latency": roofline_latency, "clocks": clocks}

    sampler = ClockSampler(local)
    if args.plan:
        w, c = (int(v) for v in args.plan.split("x"))
        _native.set_plan_override(w, c, 1)
    res = run_one(args.workload, args.steps, args.warmup, args.fused_only, args.only_mode, sampler)
    name, B, N, Dm, desc = res["name"], res["B"], res["N"], res["Dm"], res["desc"]
    head_mode, is_bary, modes, breakdown = res["head_mode"], res["is_bary"], res["modes"], res["breakdown"]
    e2e, roofline, roofline_mufu, roofline_latency = res["e2e"], res["roofline"], res["roofline_mufu"], res["roofline_latency"]
    launches, clocks = res["launches"], res["clocks"]
    head = modes[head_mode]
    # The default run also reports the other north-star shapes: the tiled
    # N = M = 4096 problem (C3) and the barycenter (C5), each timed on its own
    # (3 warm-up steps; C3 at most 10 timed steps, C5 at most 20).
    subs = {}
    if args.workload == "c2" and not args.fused_only:
        for sub, k in (("c3", 10), ("c5", 20)):
            # A failure of an extra workload (a library error raised on every
            # rank alike) is reported in its entry, not allowed to take the
            # headline line with it.
            try:
                r = run_one(sub, min(args.steps, k), 3, True, None, ClockSampler(local))
            except (RuntimeError, ValueError) as exc:
                subs[sub] = {"workload": sub, "error": f"{type(exc).__name__}: {str(exc)[:300]}"}
                continue
            hm = r["modes"][r["head_mode"]]
            subs[sub] = {"workload": f"{sub}: {r['desc']}; mode = {r['head_mode']}",
                         "value": hm["value"], "unit": "cells/s", "ms_per_step": hm["ms_per_step"],
                         "scaling": "strong" if r["is_bary"] else "weak", "kernel_ms_per_step": r["breakdown"],
                         "gpu_launches": r["launches"], "roofline_mufu": r["roofline_mufu"],
                         "roofline_latency": r["roofline_latency"], "clocks": r["clocks"]}
            if "allreduce_ms_per_step" in hm:
                subs[sub]["allreduce_ms_per_step"] = hm["allreduce_ms_per_step"]
            if "exchange_adam_ms_per_step" in hm:
                subs[sub]["exchange_adam_ms_per_step"] = hm["exchange_adam_ms_per_step"]
    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = time_oracle(name, 10.0)
        cpu_baseline = {"value": v, "unit": "cells/s", "cores": cores, "kind": "port", "sample": sample}

    if world > 1:
        # The cached barycenter graphs hold captured NCCL calls: release them
        # before the process group, whose teardown otherwise waits on them.
        torch.cuda.synchronize(dev)
        _bc.clear_graph_cache()
        dist.destroy_process_group()
    if rank != 0:
        return
    pub = PUBLISHED.get(name, {}).get(head_mode)
    line = {
        "metric": "fwd+bwd DP cells/s", "value": head["value"], "unit": "cells/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "strong" if is_bary else "weak",
        "vs_baseline": (head["value"] / world / pub) if pub else None,
        "dtype": "f32", "data": "synthetic, seeded (BASELINE config shapes and distributions)",
        "config": {"workload": f"{name}: {desc}; headline mode = {head_mode}",
                   "global_batch": B if is_bary else B * world, "seq_len": N, "dim": Dm,
                   "parallelism": (f"dp{world} (sequence-sharded barycenter, peer-memory sum over ranks per step)" if is_bary
                                   else f"dp{world} (batch-sharded, no collective)"),
                   "l2": ("per-iteration working set (about 1 GB of tables) larger than the 126 MB L2" if is_bary else
                          "flushed before every timed step (256 MiB write, outside the events)"),
                   "queue_warmup": "16 L2-flush writes (about 0.7 ms) queued ahead of the first timed step, outside the events",
                   "kernel_timing": ("kernel_ms_per_step and the roofline's launch durations: per-kernel CUDA events "
                                     "in a second pass of the same K steps; ms_per_step comes from the pass "
                                     "without them"),
                   "vs_baseline_basis": "per-GPU value / the reference's published number (unstated GPU)",
                   **({"forced_plan": args.plan} if args.plan else {})},
        "modes": modes,
        "kernel_ms_per_step": breakdown,
        "roofline": roofline,
        "roofline_mufu": roofline_mufu,
        "roofline_latency": roofline_latency,
        "cpu_baseline": cpu_baseline,
        "e2e": e2e,
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if subs:
        line["workloads"] = subs
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
