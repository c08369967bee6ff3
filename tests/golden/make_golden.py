"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run in a container where the reference package (BGU-CS-VIL/sdtw-cuda-torch,
Python + Numba) is importable:

    python tests/golden/make_golden.py --reference /path/to/sdtw-cuda-torch

The reference's own code computes every expected value here: its public
``SoftDTW`` module on CPU tensors (Numba CPU path, launcher.py:305-368),
its launcher functions for R and E, and ``softdtw_barycenter_cpu``.  A second
pass imports the reference's CUDA kernels (kernels.py) under the Numba CUDA
simulator (NUMBA_ENABLE_CUDASIM=1) to record what its GPU path computes at
tiny sizes: the fused direct-difference cost and the bandwidth edge case.

Inputs are seeded ``torch.randn``; every fixture is small (< 1 MB).
The GPU box never runs this script; the tests read the .npz files.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _save(name, **arrays):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    return path


def _cpu_cases():
    import torch
    from softdtw_cuda import SoftDTW, softdtw_barycenter_cpu
    from softdtw_cuda.distances import sqeuclidean
    from softdtw_cuda.cuda.launcher import softdtw_forward_cpu, softdtw_backward_cpu

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    manifest = {}

    def run(name, B, N, M, Dm, gamma, *, bandwidth=None, normalize=False, dtype=torch.float32,
            seed=0, reduction="sum", save_tables=True):
        torch.manual_seed(seed)
        x = torch.randn(B, N, Dm, dtype=dtype)
        y = torch.randn(B, M, Dm, dtype=dtype)
        xr = x.clone().requires_grad_(True)
        yr = y.clone().requires_grad_(True)
        mod = SoftDTW(gamma=gamma, bandwidth=bandwidth, normalize=normalize, fused=False)
        out = mod(xr, yr)
        loss = out.sum() if reduction == "sum" else out.mean()
        loss.backward()
        arrays = dict(x=x.numpy(), y=y.numpy(), out=out.detach().numpy(),
                      grad_x=xr.grad.numpy(), grad_y=yr.grad.numpy())
        if save_tables and not normalize:
            D = sqeuclidean(x, y)
            bw = -1.0 if bandwidth is None or bandwidth <= 0 else float(bandwidth)
            o2, R = softdtw_forward_cpu(D, float(gamma), bw)
            E = softdtw_backward_cpu(D, R, float(gamma), bw)
            arrays.update(D=D.numpy(), R=R.numpy(), E=E.numpy())
        _save(name, **arrays)
        manifest[name] = dict(B=B, N=N, M=M, Dim=Dm, gamma=gamma, bandwidth=bandwidth,
                              normalize=normalize, dtype=str(dtype).replace("torch.", ""),
                              seed=seed, reduction=reduction, tables=bool(save_tables and not normalize))

    # BASELINE config 1 (CPU-runnable reference check) and a gamma sweep on it.
    run("c1", 4, 64, 64, 3, 1.0)
    run("c1_g0p01", 4, 64, 64, 3, 0.01)
    run("c1_g0p1", 4, 64, 64, 3, 0.1)
    run("c1_g10", 4, 64, 64, 3, 10.0)
    run("c1_mean", 4, 64, 64, 3, 1.0, reduction="mean")
    # Ragged / unequal / degenerate lengths.
    run("uneq", 2, 12, 9, 3, 1.0)
    run("tiny_1x1", 1, 1, 1, 2, 1.0)
    run("tiny_1x7", 2, 1, 7, 3, 1.0)
    run("tiny_5x1", 2, 5, 1, 3, 1.0)
    run("odd_33x70", 3, 33, 70, 5, 0.5, seed=3)
    # Sakoe-Chiba bandwidth.
    run("bw2", 2, 10, 10, 3, 1.0, bandwidth=2.0)
    run("bw3_uneq", 2, 12, 9, 3, 1.0, bandwidth=3.0, seed=1)
    # normalize=True (concatenation trick, module.py:99-111).
    run("norm", 2, 10, 10, 3, 1.0, normalize=True)
    run("norm_g0p1", 3, 24, 24, 4, 0.1, normalize=True, seed=2)
    # float64 pipeline.
    run("f64", 1, 6, 5, 2, 1.0, dtype=torch.float64)
    run("f64_mid", 2, 40, 31, 3, 0.1, dtype=torch.float64, seed=5)
    # Mid-size shape (loss and gradients only).
    run("mid", 4, 128, 128, 16, 1.0, seed=7, save_tables=False)

    # Barycenter (barycenters.py:17-229) on CPU, no early stopping.
    torch.manual_seed(11)
    t = torch.linspace(0, 1, 20)
    base = torch.stack([torch.sin(6.28 * t), torch.cos(6.28 * t)], -1)
    X = base[None] + 0.2 * torch.randn(16, 20, 2)
    bary = softdtw_barycenter_cpu(X, gamma=1.0, max_iter=10, lr=0.1, early_stopping=False)
    w = torch.rand(16) + 0.5
    bary_w = softdtw_barycenter_cpu(X, gamma=1.0, weights=w, max_iter=10, lr=0.1,
                                    early_stopping=False)
    _save("bary", X=X.numpy(), bary=bary.numpy(), weights=w.numpy(), bary_w=bary_w.numpy())
    manifest["bary"] = dict(gamma=1.0, max_iter=10, lr=0.1, early_stopping=False)
    return manifest


_SIM_SNIPPET = r"""
import json, math, sys
import numpy as np
from softdtw_cuda.cuda import kernels as K

out = {}
rng = np.random.default_rng(0)

# Fused forward/backward kernels (kernels.py:7-122) driven diagonal by diagonal
# the way launcher.py:65-84 and :139-158 drive them.
B, N, M, Dm, gamma = 2, 7, 5, 3, 1.0
X = rng.standard_normal((B, N, Dm)).astype(np.float32)
Y = rng.standard_normal((B, M, Dm)).astype(np.float32)
R = np.full((B, N + 2, M + 2), np.inf, dtype=np.float32); R[:, 0, 0] = 0.0
for p in range(N + M - 1):
    i_min = max(0, p - (M - 1)); i_max = min(N - 1, p)
    if i_max < i_min: continue
    L = i_max - i_min + 1
    K.softdtw_forward_diag_sqeuclid_cuda[(1, B), 32](X, Y, R, gamma, -1.0, N, M, Dm, p)
Rw = R.copy(); Rw[:, :, -1] = -np.inf; Rw[:, -1, :] = -np.inf; Rw[:, -1, -1] = Rw[:, -2, -2]
logE = np.full((B, N + 2, M + 2), -np.inf, dtype=np.float32); logE[:, -1, -1] = 0.0
for p in range(N + M - 2, -1, -1):
    K.softdtw_backward_log_diag_sqeuclid_cuda[(1, B), 32](X, Y, Rw, logE, 1.0 / gamma, -1.0, N, M, Dm, p)
E = np.exp(logE[:, 1:N + 1, 1:M + 1])
np.savez_compressed(sys.argv[1] + "/sim_fused.npz", x=X, y=Y, R=R, E=E)
fused_nan = int(np.isnan(E).sum())

# D-input single-block kernels (kernels.py:126-149, 226-265) with a bandwidth,
# driven as launcher.py:185 and :257 drive them: records the GPU-path NaNs.
B, N, M, bw, gamma = 1, 6, 6, 1.0, 1.0
D = (rng.standard_normal((B, N, M)) ** 2).astype(np.float32)
R = np.full((B, N + 2, M + 2), np.inf, dtype=np.float32); R[:, 0, 0] = 0.0
tpb = max(N, M); n_passes = 2 * tpb - 1
K.softdtw_forward_kernel[B, tpb](D, gamma, bw, N, M, n_passes, R)
Dp = np.zeros((B, N + 2, M + 2), dtype=np.float32); Dp[:, 1:N + 1, 1:M + 1] = D
Rw = R.copy(); Rw[:, :, -1] = -np.inf; Rw[:, -1, :] = -np.inf; Rw[:, -1, -1] = Rw[:, -2, -2]
logE = np.full((B, N + 2, M + 2), -np.inf, dtype=np.float32); logE[:, -1, -1] = 0.0
K.softdtw_backward_log_cuda[B, tpb](Dp, Rw, 1.0 / gamma, bw, N, M, n_passes, logE)
E = np.exp(logE[:, 1:N + 1, 1:M + 1])
np.savez_compressed(sys.argv[1] + "/sim_bw_gpu.npz", D=D, R=R, E=E, bandwidth=bw, gamma=gamma)
print(json.dumps({"sim_fused_nan": fused_nan, "sim_bw_gpu_nan": int(np.isnan(E).sum())}))
"""


def _sim_cases(reference: str):
    env = dict(os.environ)
    env["NUMBA_ENABLE_CUDASIM"] = "1"
    env["PYTHONPATH"] = reference + os.pathsep + env.get("PYTHONPATH", "")
    res = subprocess.run([sys.executable, "-c", _SIM_SNIPPET, HERE], env=env, check=True,
                         capture_output=True, text=True)
    return json.loads(res.stdout.strip().splitlines()[-1])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    manifest = _cpu_cases()
    manifest["_sim"] = _sim_cases(os.path.abspath(args.reference))
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print(json.dumps(manifest["_sim"]))


if __name__ == "__main__":
    main()
