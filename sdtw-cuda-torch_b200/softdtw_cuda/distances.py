"""Pairwise cost between sequences (softdtw_cuda/distances.py:6-35).

``sqeuclidean`` returns D[b,i,j] = ||x[b,i] - y[b,j]||^2 as
||x||^2 + ||y||^2 - 2 x.y^T clamped at zero.  On CUDA float tensors the cost
matrix and its gradient come from libsdtw_b200 kernels; other tensors use the
same expression in plain torch ops.
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from . import _native

_SQEUCLID_NAMES = ("sqeuclidean", "sq_euclidean", "squared_euclidean")
_KERNEL_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


class _SqEuclideanCUDA(Function):
    """Cost matrix on the device; backward = 2(x rowsum(G) - G y), 2(y colsum(G) - G^T x),
    with G zeroed where the clamp at 0 was active."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, y: torch.Tensor):
        D = _native.cost_sqeuclid(x, y, direct=False)
        ctx.save_for_backward(x, y, D)
        return D.to(x.dtype)

    @staticmethod
    def backward(ctx, grad_D: torch.Tensor):
        x, y, D = ctx.saved_tensors
        gx, gy = _native.grad_sqeuclid(grad_D, D, x, y, ctx.needs_input_grad[0], ctx.needs_input_grad[1])
        return (None if gx is None else gx.to(x.dtype)), (None if gy is None else gy.to(y.dtype))


def _sqeuclidean_torch(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    x2 = (x * x).sum(dim=-1)
    y2 = (y * y).sum(dim=-1)
    xy = torch.bmm(x, y.transpose(1, 2))
    D = x2.unsqueeze(2) + y2.unsqueeze(1) - 2.0 * xy
    return D.clamp_min(0.0)


def sqeuclidean(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """Squared Euclidean cost D (B,N,M) of x (B,N,D) and y (B,M,D)."""
    if x.dim() != 3 or y.dim() != 3:
        raise ValueError(f"Expected x,y as (B,N,D)/(B,M,D). Got {tuple(x.shape)} and {tuple(y.shape)}")
    if x.shape[0] != y.shape[0] or x.shape[2] != y.shape[2]:
        raise ValueError(f"Batch/features mismatch: {tuple(x.shape)} vs {tuple(y.shape)}")
    if (x.is_cuda and y.is_cuda and x.device == y.device and x.dtype in _KERNEL_DTYPES
            and y.dtype == x.dtype and x.numel() > 0 and y.numel() > 0):
        return _SqEuclideanCUDA.apply(x, y)
    return _sqeuclidean_torch(x, y)


def pairwise_distance(x: torch.Tensor, y: torch.Tensor, *, dist: str) -> torch.Tensor:
    dist = dist.lower()
    if dist in _SQEUCLID_NAMES:
        return sqeuclidean(x, y)
    raise ValueError(f"Unknown dist='{dist}'. Supported: 'sqeuclidean'")
