"""Fused squared-Euclidean Soft-DTW on x, y (softdtw_cuda/autograd_xy.py:12-51).

``SoftDTWXYAutograd.apply(X, Y, gamma, bandwidth)`` computes the cost
sum_k (x_ik - y_jk)^2 inside the library (no cost tensor is returned to the
caller) and its backward returns dL/dX and dL/dY directly:
    grad_X = 2 (X * rowsum(G) - G Y),  grad_Y = 2 (Y * colsum(G) - G^T X),
G = grad_out[b] * E[b].  CUDA only, as in the reference.  float64 inputs take
the library's float64 device path (cost, forward, backward and this chain rule
in double).
"""
from __future__ import annotations

import torch
from torch.autograd import Function

from . import _native
from .autograd import _normalize_bandwidth


class SoftDTWXYAutograd(Function):
    @staticmethod
    def forward(ctx, X: torch.Tensor, Y: torch.Tensor, gamma: float, bandwidth: float | None):
        if not (X.is_cuda and Y.is_cuda):
            raise ValueError("Expected CUDA tensors X and Y")
        if X.dim() != 3 or Y.dim() != 3:
            raise ValueError(f"Expected X,Y as (B,N,D)/(B,M,D). Got {tuple(X.shape)} and {tuple(Y.shape)}")
        if X.shape[0] != Y.shape[0] or X.shape[2] != Y.shape[2]:
            raise ValueError(f"Batch/features mismatch: {tuple(X.shape)} vs {tuple(Y.shape)}")
        gamma_f = float(gamma)
        bw = _normalize_bandwidth(bandwidth)
        ctx.f64 = X.dtype == torch.float64 or Y.dtype == torch.float64
        if ctx.f64:
            D = _native.cost_sqeuclid_f64(X, Y)
            out, R = _native.forward_f64(D, gamma_f, bw)
            ctx.save_for_backward(X, Y, D, R)
            ctx.gamma = gamma_f
            ctx.bandwidth = bw
            return out.to(X.dtype)
        out, score = _native.forward_xy(X, Y, gamma_f, bw)
        ctx.save_for_backward(X, Y, score)
        ctx.gamma = gamma_f
        ctx.bandwidth = bw
        return out.to(X.dtype)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        if ctx.f64:
            X, Y, D, R = ctx.saved_tensors
            G = _native.backward_f64(D, R, grad_output, ctx.gamma, ctx.bandwidth)
            gx, gy = _native.grad_sqeuclid_f64(G, X, Y, ctx.needs_input_grad[0], ctx.needs_input_grad[1])
            return (None if gx is None else gx.to(X.dtype)), (None if gy is None else gy.to(Y.dtype)), None, None
        X, Y, score = ctx.saved_tensors
        gx, gy = _native.backward_xy(X, Y, score, grad_output, ctx.gamma, ctx.bandwidth,
                                     need_x=ctx.needs_input_grad[0], need_y=ctx.needs_input_grad[1])
        return (None if gx is None else gx.to(X.dtype)), (None if gy is None else gy.to(Y.dtype)), None, None


class SoftDTWXYNormAutograd(Function):
    """The fused normalized triple: ``apply(X, Y, gamma, bandwidth)`` returns
    the 3B losses [SoftDTW(x_b, y_b) | SoftDTW(x_b, x_b) | SoftDTW(y_b, y_b)]
    of softdtw_cuda/module.py:99-111, with x and y read in place instead of
    concatenated; the backward folds the self pairs' gradients into dL/dX and
    dL/dY.  float32 CUDA tensors (bf16/fp16 are computed in float32)."""

    @staticmethod
    def forward(ctx, X: torch.Tensor, Y: torch.Tensor, gamma: float, bandwidth: float | None):
        gamma_f = float(gamma)
        bw = _normalize_bandwidth(bandwidth)
        out, score = _native.forward_xy_norm(X, Y, gamma_f, bw)
        ctx.save_for_backward(X, Y, score)
        ctx.gamma = gamma_f
        ctx.bandwidth = bw
        return out.to(X.dtype)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        X, Y, score = ctx.saved_tensors
        gx, gy = _native.backward_xy_norm(X, Y, score, grad_output, ctx.gamma, ctx.bandwidth)
        return (gx.to(X.dtype) if ctx.needs_input_grad[0] else None,
                gy.to(Y.dtype) if ctx.needs_input_grad[1] else None, None, None)
