"""Launcher-level functions with the reference's signatures
(softdtw_cuda/cuda/launcher.py:33-368).

They return and accept the R table in the reference layout (B, N+2, M+2),
converting from/to the library's score table, so code that called the
reference launchers directly keeps working.  The autograd Functions do not go
through here: the x/y pairs they call keep each cell's predecessor weights
instead, which is all their backward needs.
"""
from __future__ import annotations

import torch

from .. import _native


def _bw(bandwidth: float) -> float:
    bw = float(bandwidth)
    return -1.0 if bw <= 0 else bw


def softdtw_forward_cuda_fused_sqeuclid(X: torch.Tensor, Y: torch.Tensor, gamma: float, bandwidth: float):
    """Fused forward on CUDA X (B,N,D), Y (B,M,D): returns (out (B,), R (B,N+2,M+2))."""
    if not (X.is_cuda and Y.is_cuda):
        raise ValueError("Expected CUDA tensors X and Y")
    if X.dim() != 3 or Y.dim() != 3:
        raise ValueError(f"Expected X,Y as (B,N,D)/(B,M,D). Got {tuple(X.shape)} and {tuple(Y.shape)}")
    if X.shape[0] != Y.shape[0] or X.shape[2] != Y.shape[2]:
        raise ValueError(f"Batch/features mismatch: {tuple(X.shape)} vs {tuple(Y.shape)}")
    B, N, _ = X.shape
    M = Y.shape[1]
    # The x/y forward keeps predecessor weights, not scores, for its backward;
    # the R table comes from the scores of the same direct-form cost.
    D = _native.cost_sqeuclid(X, Y, direct=True)
    out, score = _native.forward(D, gamma, _bw(bandwidth))
    R = _native.score_to_R(score, B, N, M, gamma)
    return out.to(X.dtype), R.to(X.dtype)


def softdtw_backward_cuda_fused_sqeuclid(X: torch.Tensor, Y: torch.Tensor, R: torch.Tensor, gamma: float,
                                         bandwidth: float) -> torch.Tensor:
    """E (B,N,M) = dR[N,M]/dD from the fused forward's R table."""
    if not (X.is_cuda and Y.is_cuda and R.is_cuda):
        raise ValueError("Expected CUDA tensors X, Y, R")
    if X.dim() != 3 or Y.dim() != 3:
        raise ValueError(f"Expected X,Y as (B,N,D)/(B,M,D). Got {tuple(X.shape)} and {tuple(Y.shape)}")
    if X.shape[0] != Y.shape[0] or X.shape[2] != Y.shape[2]:
        raise ValueError(f"Batch/features mismatch: {tuple(X.shape)} vs {tuple(Y.shape)}")
    B, N, _ = X.shape
    M = Y.shape[1]
    if tuple(R.shape) != (B, N + 2, M + 2):
        raise ValueError(f"Expected R shape {(B, N + 2, M + 2)}, got {tuple(R.shape)}")
    score = _native.R_to_score(R, gamma)
    return _native.backward(score, None, B, N, M, gamma, _bw(bandwidth)).to(X.dtype)


def softdtw_forward_cuda(D: torch.Tensor, gamma: float, bandwidth: float):
    """Forward on a CUDA cost matrix: (out (B,), R (B,N+2,M+2))."""
    if not D.is_cuda:
        raise ValueError("Expected CUDA tensor D")
    if gamma <= 0:
        raise ValueError(f"gamma must be > 0, got {gamma}")
    B, N, M = D.shape
    out, score = _native.forward(D, gamma, _bw(bandwidth))
    R = _native.score_to_R(score, B, N, M, gamma)
    return out.to(D.dtype), R.to(D.dtype)


def softdtw_backward_cuda_log(D: torch.Tensor, R: torch.Tensor, gamma: float, bandwidth: float) -> torch.Tensor:
    """E (B,N,M) = dR[N,M]/dD for a CUDA cost matrix and its forward R table."""
    if not D.is_cuda:
        raise ValueError("Expected CUDA tensor D")
    if gamma <= 0:
        raise ValueError(f"gamma must be > 0, got {gamma}")
    B, N, M = D.shape
    score = _native.R_to_score(R, gamma)
    return _native.backward(score, None, B, N, M, gamma, _bw(bandwidth)).to(D.dtype)


def softdtw_forward_cpu(D: torch.Tensor, gamma: float, bandwidth: float):
    """Host forward: (out (B,), R (B,N+2,M+2)) in D's dtype."""
    out, R = _native.cpu_forward(D, gamma, _bw(bandwidth))
    return out.to(device=D.device, dtype=D.dtype), R.to(device=D.device, dtype=D.dtype)


def softdtw_backward_cpu(D: torch.Tensor, R: torch.Tensor, gamma: float, bandwidth: float) -> torch.Tensor:
    """Host backward: E (B,N,M) in D's dtype."""
    E = _native.cpu_backward(R, None, gamma, _bw(bandwidth))
    return E.to(device=D.device, dtype=D.dtype).contiguous()
