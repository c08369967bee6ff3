"""Soft-DTW barycenters (softdtw_cuda/barycenters.py:17-229).

The barycenter b (N,D) minimises sum_i w_i SoftDTW(b, X_i) by Adam with
gradient-norm clipping at 1.0 and cosine learning-rate annealing to lr/10;
optional early stopping on absolute loss improvement after half of max_iter
(the method of Cuturi & Blondel, ICML 2017).  Behaviour, defaults and
progress messages follow the reference.  The multi-GPU version is
``softdtw_cuda.distributed.sharded_barycenter``.
"""
from __future__ import annotations

import time

import torch

from .module import SoftDTW


def softdtw_barycenter(
    X: torch.Tensor,
    *,
    gamma: float = 1.0,
    weights: torch.Tensor | None = None,
    max_iter: int = 100,
    lr: float = 0.1,
    init: torch.Tensor | None = None,
    device: str | torch.device | None = None,
    verbose: bool = False,
    fused: bool | None = None,
    early_stopping: bool = True,
    patience: int = 10,
    tol: float = 1e-5,
) -> torch.Tensor:
    """Barycenter (N, D) of X (B, N, D) under Soft-DTW.

    weights: (B,) non-negative, normalised to sum 1 (uniform if None).
    init:    (N, D) starting point (the weighted mean if None).
    device:  where to optimise (X's device if None).
    fused:   None = auto, True = require the fused kernels, False = never.
    early_stopping / patience / tol: stop once the loss has not improved by
             more than `tol` (absolute) for `patience` iterations, but only
             after max_iter // 2 iterations.
    """
    device = device or X.device
    X = X.to(device)
    B, N, D = X.shape
    if weights is None:
        w = torch.full((B,), 1.0 / B, device=device)
    else:
        w = weights.to(device)
        w = w / w.sum()
    if init is None:
        bary = (X * w.view(B, 1, 1)).sum(dim=0).clone()
    else:
        bary = init.clone().to(device)
    bary.requires_grad_(True)

    loss_fn = SoftDTW(gamma=gamma, normalize=False, fused=fused)
    opt = torch.optim.Adam([bary], lr=lr)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=max_iter, eta_min=lr * 0.1)

    t0 = time.time()
    best = float("inf")
    stale = 0
    for it in range(max_iter):
        opt.zero_grad()
        d = loss_fn(bary.unsqueeze(0).expand(B, -1, -1), X)
        loss = (w * d).sum()
        loss.backward()
        torch.nn.utils.clip_grad_norm_([bary], max_norm=1.0)
        opt.step()
        sched.step()

        loss_val = loss.item()
        improvement = float("nan")
        if early_stopping:
            improvement = best - loss_val
            if improvement > tol:
                best = loss_val
                stale = 0
            else:
                stale += 1
            if stale >= patience and it > max_iter // 2:
                if verbose:
                    print(f"Early stopping at iteration {it + 1} (no improvement for {patience} iterations)")
                break

        if verbose and (it + 1) % 20 == 0:
            if torch.cuda.is_available():
                torch.cuda.synchronize()
            _ = time.time() - t0
            lr_val = opt.param_groups[0]["lr"]
            imp = f"{improvement:9.6f}" if early_stopping else "     N/A "
            print(f"Iteration {it + 1:3d}/{max_iter} | Loss: {loss_val:9.6f} | Improvement: {imp} | LR: {lr_val:.2e}")

    return bary.detach()


def softdtw_barycenter_cpu(
    X: torch.Tensor,
    *,
    gamma: float = 1.0,
    weights: torch.Tensor | None = None,
    max_iter: int = 100,
    lr: float = 0.1,
    init: torch.Tensor | None = None,
    verbose: bool = False,
    fused: bool | None = None,
    early_stopping: bool = True,
    patience: int = 10,
    tol: float = 1e-5,
) -> torch.Tensor:
    """``softdtw_barycenter`` with device="cpu"."""
    return softdtw_barycenter(X, gamma=gamma, weights=weights, max_iter=max_iter, lr=lr, init=init,
                              device="cpu", verbose=verbose, fused=fused, early_stopping=early_stopping,
                              patience=patience, tol=tol)
