"""Soft-DTW on an arbitrary cost matrix D (softdtw_cuda/autograd.py:11-48).

``SoftDTWAutograd.apply(D, gamma, bandwidth)`` returns R[N,M] per batch
element; its backward returns grad_D = grad_out[b] * E[b] where E is the
expected alignment matrix.  CUDA tensors use the libsdtw_b200 wavefront kernels
(float32 arithmetic; float16/bfloat16 inputs are computed in float32; float64
inputs take the library's float64 device path, in double throughout), CPU
tensors the library's double-precision host implementation.
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from . import _native
from .utils.checks import check_D


def _normalize_bandwidth(bandwidth) -> float:
    # None or <= 0 disables the band (autograd.py:19-23).
    if bandwidth is None:
        return -1.0
    bw = float(bandwidth)
    return -1.0 if bw <= 0 else bw


class SoftDTWAutograd(Function):
    @staticmethod
    def forward(ctx, D: torch.Tensor, gamma: float, bandwidth: float | None):
        check_D(D)
        gamma_f = float(gamma)
        if gamma_f <= 0:
            raise ValueError(f"gamma must be > 0, got {gamma_f}")
        bw = _normalize_bandwidth(bandwidth)
        B, N, M = D.shape
        ctx.f64 = D.is_cuda and D.dtype == torch.float64
        if ctx.f64:
            out, table = _native.forward_f64(D, gamma_f, bw)
            ctx.save_for_backward(table, D.detach())
        elif D.is_cuda:
            out, table = _native.forward(D, gamma_f, bw)
            ctx.save_for_backward(table)
        else:
            out, table = _native.cpu_forward(D, gamma_f, bw)
            ctx.save_for_backward(table)
        ctx.gamma = gamma_f
        ctx.bandwidth = bw
        ctx.dims = (B, N, M)
        ctx.cuda = D.is_cuda
        ctx.dtype = D.dtype
        return out.to(D.dtype)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        B, N, M = ctx.dims
        if ctx.f64:
            table, D = ctx.saved_tensors
            return _native.backward_f64(D, table, grad_output, ctx.gamma, ctx.bandwidth), None, None
        (table,) = ctx.saved_tensors
        if ctx.cuda:
            E = _native.backward(table, grad_output, B, N, M, ctx.gamma, ctx.bandwidth)
        else:
            E = _native.cpu_backward(table, grad_output, ctx.gamma, ctx.bandwidth)
        return E.to(ctx.dtype), None, None


class SoftDTWSqEuclidAutograd(Function):
    """Unfused squared-Euclidean Soft-DTW on CUDA float tensors.

    Computes the same quantity as ``SoftDTWAutograd.apply(sqeuclidean(X, Y), ...)``
    (softdtw_cuda/module.py:116-118): the cost matrix is built explicitly as
    ||x||^2 + ||y||^2 - 2 x.y clamped at 0 and kept (in the library's
    anti-diagonal layout) for the backward, whose chain rule to X and Y zeroes
    the cells where the clamp was active, as torch autograd of
    distances.py:20-28 does.
    """

    @staticmethod
    def forward(ctx, X: torch.Tensor, Y: torch.Tensor, gamma: float, bandwidth: float | None):
        gamma_f = float(gamma)
        if gamma_f <= 0:
            raise ValueError(f"gamma must be > 0, got {gamma_f}")
        bw = _normalize_bandwidth(bandwidth)
        out, score, cost = _native.forward_sqeuclid(X, Y, gamma_f, bw)
        ctx.save_for_backward(X, Y, score, cost)
        ctx.gamma = gamma_f
        ctx.bandwidth = bw
        return out.to(X.dtype)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        X, Y, score, cost = ctx.saved_tensors
        gx, gy = _native.backward_sqeuclid(X, Y, score, cost, grad_output, ctx.gamma, ctx.bandwidth,
                                           need_x=ctx.needs_input_grad[0], need_y=ctx.needs_input_grad[1])
        return (None if gx is None else gx.to(X.dtype)), (None if gy is None else gy.to(Y.dtype)), None, None


class SoftDTWSqEuclidNormAutograd(Function):
    """The unfused normalized triple: the 3B losses [xy | xx | yy] of
    softdtw_cuda/module.py:99-111 on the clamped expanded cost, x and y read
    in place instead of concatenated; the backward folds the self pairs'
    gradients into dL/dX and dL/dY."""

    @staticmethod
    def forward(ctx, X: torch.Tensor, Y: torch.Tensor, gamma: float, bandwidth: float | None):
        gamma_f = float(gamma)
        if gamma_f <= 0:
            raise ValueError(f"gamma must be > 0, got {gamma_f}")
        bw = _normalize_bandwidth(bandwidth)
        out, score, cost = _native.forward_sqeuclid_norm(X, Y, gamma_f, bw)
        ctx.save_for_backward(X, Y, score, cost)
        ctx.gamma = gamma_f
        ctx.bandwidth = bw
        return out.to(X.dtype)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        X, Y, score, cost = ctx.saved_tensors
        gx, gy = _native.backward_sqeuclid_norm(X, Y, score, cost, grad_output, ctx.gamma, ctx.bandwidth)
        return (gx.to(X.dtype) if ctx.needs_input_grad[0] else None,
                gy.to(Y.dtype) if ctx.needs_input_grad[1] else None, None, None)
