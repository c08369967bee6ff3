#!/usr/bin/env python
"""Soft-DTW forward+backward DP-cell throughput on B200.

Workload: per GPU B=32, N=M=512, D=64 float32 x, y ~ N(0,1)
(seeded, synthetic), gamma=1, squared-Euclidean cost;
one step = SoftDTW(fused=...)(x, y).mean().backward() producing dL/dx and dL/dy.
Metric: DP cells per second, cells = B*N*M per step, summed over all GPUs
(weak scaling: every rank runs its own B=32 batch; no collective on the path).
The headline `value` is the default CUDA path (fused=None -> fused); the
unfused path is reported under "modes".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`--impl reference` times the reference's CPU algorithm (the oracle port in
oracle/, all host threads) on the same workload.
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

WORKLOADS = {
    # name: (B, N, M, D, gamma, description)
    "c2": (32, 512, 512, 64, 1.0, "BASELINE config 2: B=32/GPU, N=M=512, D=64, gamma=1, fwd+bwd, mean reduction"),
    "c3": (16, 4096, 4096, 8, 0.1, "BASELINE config 3 shape: B=16/GPU, N=M=4096, D=8, gamma=0.1, fwd+bwd"),
    "c4a": (64, 1024, 768, 128, 1.0, "BASELINE config 4a: B=64/GPU, N=1024, M=768, D=128, gamma=1"),
}
PUBLISHED = {  # reference, B=32 N=M=512 D=64 fwd+bwd (unstated GPU)
    "c2": {"fused": 32 * 512 * 512 / 0.14136, "unfused": 32 * 512 * 512 / 0.02010},
}
MUFU_PER_CELL = 7          # algorithmic ex2/lg2 per DP cell, forward + backward (reference algorithm)
MUFU_PER_SM_CLK = 16       # ex2/lg2 results per SM per clock
# Algorithmic HBM bytes per DP cell of each library kernel: every table entry
# read or written once (cost 4 B, score 8 B as a (hi, lo) pair, E 4 B).
ALG_BYTES = {"cost_wl": 4, "wavefront_fwd": 12, "wavefront_bwd": 12, "wl_to_rm": 8, "grad_xy": 8,
             "rm_to_wl": 8, "cost_rowmajor": 4}
# Algorithmic MUFU ops per cell of the reference algorithm: forward softmin
# (2 ex2 + 1 lg2), reverse log-sum-exp (2 ex2 + 1 lg2) and E = exp(log E) (1 ex2).
ALG_MUFU = {"wavefront_fwd": 3, "wavefront_bwd": 4}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    # Profiling runs: only the fused timed steps (no unfused mode, no end-to-end leg).
    ap.add_argument("--fused-only", action="store_true")
    return ap.parse_args()


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


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    import numpy as np
    import torch

    from oracle import oracle as O

    B, N, M, Dm, gamma, desc = WORKLOADS[args.workload]
    torch.manual_seed(1234)
    x = torch.randn(B, N, Dm).numpy()
    y = torch.randn(B, M, Dm).numpy()
    g = np.full(B, 1.0 / B)
    cores = O.num_threads()
    for _ in range(args.warmup):
        O.loss_and_grads(x, y, gamma=gamma, grad_out=g)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.loss_and_grads(x, y, gamma=gamma, grad_out=g)
        times.append(time.perf_counter() - t0)
    cells = B * N * M
    ms = 1e3 * statistics.mean(times)
    value = cells / (ms / 1e3)
    line = {
        "impl": "reference", "metric": "fwd+bwd DP cells/s", "value": value, "unit": "cells/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (f64 DP)",
        "data": "synthetic N(0,1), seeded",
        "config": {"workload": desc + " (CPU: unfused, the reference has no CPU fused mode)",
                   "global_batch": B, "seq_len": N, "dim": Dm, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "cells/s", "cores": cores, "kind": "port",
                         "sample": f"full batch ({B}x{N}x{M}, D={Dm}) per step; oracle/ restatement of "
                                   "launcher.py:305-368 + numpy cost and chain rule"},
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

    B, N, M, Dm, gamma, desc = WORKLOADS[args.workload]
    cells = B * N * M
    gen = torch.Generator().manual_seed(1234 + rank)
    x_h = torch.randn(B, N, Dm, generator=gen).pin_memory()
    y_h = torch.randn(B, M, Dm, generator=gen).pin_memory()
    x = x_h.to(dev)
    y = y_h.to(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > 126 MB L2

    def step(fused):
        xr = x.detach().requires_grad_(True)
        yr = y.detach().requires_grad_(True)
        out = SoftDTW(gamma=gamma, fused=fused)(xr, yr)
        out.mean().backward()
        return xr.grad, yr.grad

    sampler = ClockSampler(local)

    def timed(fn, k):
        times = []
        stream = torch.cuda.current_stream(dev)
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

    modes = {}
    launches = 0
    breakdown = {}
    with sampler:
        for name, fused in (("fused", None), ("unfused", False))[:1 if args.fused_only else 2]:
            for _ in range(args.warmup):
                step(fused)
            torch.cuda.synchronize(dev)
            barrier()
            torch.cuda.synchronize(dev)
            l0 = _native.launch_count
            if name == "fused":
                _native.timing_enable(True)  # per-kernel CUDA events on the launching stream
            ms = timed(lambda: step(fused), args.steps)
            if name == "fused":
                launches = _native.launch_count - l0
                kt = _native.timing_read()
                _native.timing_enable(False)
                breakdown = {k: v[0] / max(v[1], 1) * (v[1] / args.steps) for k, v in kt.items()}
                per_launch = {k: v[0] / max(v[1], 1) for k, v in kt.items()}
            torch.cuda.synchronize(dev)
            barrier()
            _native.check_status(dev)
            mean_ms = max_over_ranks(statistics.mean(ms))
            modes[name] = {"value": world * cells / (mean_ms / 1e3), "ms_per_step": mean_ms,
                           "median_ms": statistics.median(ms)}
            pub = PUBLISHED.get(args.workload, {}).get(name)
            modes[name]["vs_published"] = (modes[name]["value"] / world / pub) if pub else None

    # End to end through the public API with host buffers.
    gx_h = torch.empty_like(x_h).pin_memory()
    gy_h = torch.empty_like(y_h).pin_memory()
    loss_h = torch.empty((), dtype=torch.float32).pin_memory()

    def e2e_step():
        xd = x_h.to(dev, non_blocking=True).requires_grad_(True)
        yd = y_h.to(dev, non_blocking=True).requires_grad_(True)
        loss = SoftDTW(gamma=gamma)(xd, yd).mean()
        loss.backward()
        loss_h.copy_(loss.detach(), non_blocking=True)
        gx_h.copy_(xd.grad, non_blocking=True)
        gy_h.copy_(yd.grad, non_blocking=True)

    e2e_ms = float("nan")
    if not args.fused_only:
        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = max_over_ranks(statistics.mean(timed(e2e_step, args.steps)))
    h2d = x_h.numel() * 4 + y_h.numel() * 4
    d2h = 4 + gx_h.numel() * 4 + gy_h.numel() * 4

    clocks = sampler.summary()
    head = modes["fused"]

    # Roofline of the dominant kernel (largest device time per step).
    dom = max(breakdown, key=breakdown.get)
    dom_ms = per_launch[dom]
    alg_bytes = ALG_BYTES[dom] * cells
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic_c2.json")) as f:
            traffic = json.load(f).get(dom)
    except (OSError, ValueError):
        pass
    achieved = alg_bytes / (dom_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "traffic": traffic,
                "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                "alg_bytes_per_cell": ALG_BYTES[dom]}
    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    sm_mhz = clocks.get("sm_mhz") or peaks.get("sm_max_mhz", 1965.0)
    mufu_peak = n_sm * MUFU_PER_SM_CLK * sm_mhz * 1e6
    step_mufu = MUFU_PER_CELL * cells / (head["ms_per_step"] / 1e3)
    wf = {k: ALG_MUFU[k] * cells / (per_launch[k] / 1e3) for k in ALG_MUFU if k in per_launch}
    roofline_mufu = {"bound": "mufu", "unit": "Gop/s", "peak": mufu_peak / 1e9,
                     "peak_basis": f"{n_sm} SMs x {MUFU_PER_SM_CLK} ex2/lg2 per clk x {sm_mhz:.0f} MHz (median under load)",
                     "step_achieved": step_mufu / 1e9, "step_frac": step_mufu / mufu_peak,
                     "kernels": {k: {"achieved": v / 1e9, "frac": v / mufu_peak, "ms": per_launch[k],
                                     "alg_ops_per_cell": ALG_MUFU[k]} for k, v in wf.items()},
                     "alg_ops_per_cell": MUFU_PER_CELL}

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import numpy as np
        from oracle import oracle as O
        xn, yn = x_h.numpy(), y_h.numpy()
        g = np.full(B, 1.0 / B)
        O.loss_and_grads(xn, yn, gamma=gamma, grad_out=g)  # warm
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0 and reps < 200:
            O.loss_and_grads(xn, yn, gamma=gamma, grad_out=g)
            reps += 1
        dt = time.perf_counter() - t0
        cpu_baseline = {"value": reps * cells / dt, "unit": "cells/s", "cores": O.num_threads(), "kind": "port",
                        "sample": f"{reps} x full batch ({B}x{N}x{M}, D={Dm}) fwd+bwd, unfused reference "
                                  f"algorithm (oracle/), {dt:.1f} s"}

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    pub = PUBLISHED.get(args.workload, {}).get("fused")
    line = {
        "metric": "fwd+bwd DP cells/s", "value": head["value"], "unit": "cells/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (head["value"] / world / pub) if pub else None,
        "dtype": "f32", "data": "synthetic N(0,1), seeded",
        "config": {"workload": desc + "; headline = default CUDA path (fused=None -> fused)",
                   "global_batch": B * world, "seq_len": N, "dim": Dm, "parallelism": f"dp{world} (batch-sharded)",
                   "l2": "flushed before every timed step (256 MiB write, outside the events)",
                   "vs_baseline_basis": "per-GPU value / BASELINE.md published fused number (unstated GPU)"},
        "modes": modes,
        "kernel_ms_per_step": breakdown,
        "roofline": roofline,
        "roofline_mufu": roofline_mufu,
        "cpu_baseline": cpu_baseline,
        "e2e": None if args.fused_only else {
            "value": world * cells / (e2e_ms / 1e3), "unit": "cells/s", "ms_per_step": e2e_ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "api": "softdtw_cuda.SoftDTW (pinned host x,y in; loss, dL/dx, dL/dy out)"},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
