"""The library's CUDA entry points as PyTorch custom operators, for torch.compile.

``torch.compile`` cannot trace through the ctypes calls inside the autograd
Functions (softdtw_cuda/autograd*.py), so a compiled model would break its
graph at the loss.  The same calls are registered here as
``torch.ops.softdtw_cuda.*`` with fake (meta) implementations for shape
propagation and with their autograd formulas, and ``SoftDTW`` uses them while
compiling (``torch.compiler.is_compiling()``); eager calls keep the autograd
Functions.  Both routes make the same library calls.

  xy_forward / xy_backward   fused squared-Euclidean path (autograd_xy.py:12-51)
  sq_forward / sq_backward   unfused path with the cost kept in the library's
                             layout (module.py:116-118 through autograd.py)
  d_forward / d_backward     arbitrary cost matrix D (autograd.py:11-48)

Float32, float16 and bfloat16 CUDA tensors (computed in float32, results in the
input dtype).  The score (and cost) tables are flat float32 tensors in the
library's layout, sized by ``_native.score_elems`` / ``cost_elems``.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _native

_EMPTY = (0,)


def _grad_or_empty(need: bool, g, like: Tensor) -> Tensor:
    return g.to(like.dtype) if need else like.new_empty(_EMPTY)


# ----------------------------------------------------------------------------- fused x / y
@torch.library.custom_op("softdtw_cuda::xy_forward", mutates_args=(), device_types="cuda")
def xy_forward(x: Tensor, y: Tensor, gamma: float, bandwidth: float) -> tuple[Tensor, Tensor]:
    out, score = _native.forward_xy(x, y, gamma, bandwidth)
    return out.to(x.dtype), score


@xy_forward.register_fake
def _(x, y, gamma, bandwidth):
    B, N, M = x.shape[0], x.shape[1], y.shape[1]
    return x.new_empty((B,)), x.new_empty((_native.score_elems(B, N, M),), dtype=torch.float32)


@torch.library.custom_op("softdtw_cuda::xy_backward", mutates_args=(), device_types="cuda")
def xy_backward(x: Tensor, y: Tensor, score: Tensor, grad_out: Tensor, gamma: float, bandwidth: float,
                need_x: bool, need_y: bool) -> tuple[Tensor, Tensor]:
    gx, gy = _native.backward_xy(x, y, score, grad_out, gamma, bandwidth, need_x=need_x, need_y=need_y)
    return _grad_or_empty(need_x, gx, x), _grad_or_empty(need_y, gy, y)


@xy_backward.register_fake
def _(x, y, score, grad_out, gamma, bandwidth, need_x, need_y):
    return (torch.empty_like(x) if need_x else x.new_empty(_EMPTY)), (torch.empty_like(y) if need_y else y.new_empty(_EMPTY))


def _xy_setup(ctx, inputs, output):
    x, y, gamma, bandwidth = inputs
    ctx.save_for_backward(x, y, output[1])
    ctx.gamma, ctx.bandwidth = gamma, bandwidth


def _xy_backward(ctx, grad_out, _grad_score):
    x, y, score = ctx.saved_tensors
    nx, ny = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
    gx, gy = xy_backward(x, y, score, grad_out, ctx.gamma, ctx.bandwidth, nx, ny)
    return (gx if nx else None), (gy if ny else None), None, None


xy_forward.register_autograd(_xy_backward, setup_context=_xy_setup)


# ----------------------------------------------------------------------------- unfused x / y
@torch.library.custom_op("softdtw_cuda::sq_forward", mutates_args=(), device_types="cuda")
def sq_forward(x: Tensor, y: Tensor, gamma: float, bandwidth: float) -> tuple[Tensor, Tensor, Tensor]:
    out, score, cost = _native.forward_sqeuclid(x, y, gamma, bandwidth)
    return out.to(x.dtype), score, cost


@sq_forward.register_fake
def _(x, y, gamma, bandwidth):
    B, N, M = x.shape[0], x.shape[1], y.shape[1]
    return (x.new_empty((B,)), x.new_empty((_native.score_elems(B, N, M),), dtype=torch.float32),
            x.new_empty((_native.cost_elems(B, N, M),), dtype=torch.float32))


@torch.library.custom_op("softdtw_cuda::sq_backward", mutates_args=(), device_types="cuda")
def sq_backward(x: Tensor, y: Tensor, score: Tensor, cost: Tensor, grad_out: Tensor, gamma: float,
                bandwidth: float, need_x: bool, need_y: bool) -> tuple[Tensor, Tensor]:
    gx, gy = _native.backward_sqeuclid(x, y, score, cost, grad_out, gamma, bandwidth, need_x=need_x, need_y=need_y)
    return _grad_or_empty(need_x, gx, x), _grad_or_empty(need_y, gy, y)


@sq_backward.register_fake
def _(x, y, score, cost, grad_out, gamma, bandwidth, need_x, need_y):
    return (torch.empty_like(x) if need_x else x.new_empty(_EMPTY)), (torch.empty_like(y) if need_y else y.new_empty(_EMPTY))


def _sq_setup(ctx, inputs, output):
    x, y, gamma, bandwidth = inputs
    ctx.save_for_backward(x, y, output[1], output[2])
    ctx.gamma, ctx.bandwidth = gamma, bandwidth


def _sq_backward(ctx, grad_out, _grad_score, _grad_cost):
    x, y, score, cost = ctx.saved_tensors
    nx, ny = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
    gx, gy = sq_backward(x, y, score, cost, grad_out, ctx.gamma, ctx.bandwidth, nx, ny)
    return (gx if nx else None), (gy if ny else None), None, None


sq_forward.register_autograd(_sq_backward, setup_context=_sq_setup)


# ----------------------------------------------------------------------------- arbitrary D
@torch.library.custom_op("softdtw_cuda::d_forward", mutates_args=(), device_types="cuda")
def d_forward(D: Tensor, gamma: float, bandwidth: float) -> tuple[Tensor, Tensor]:
    out, score = _native.forward(D, gamma, bandwidth)
    return out.to(D.dtype), score


@d_forward.register_fake
def _(D, gamma, bandwidth):
    B, N, M = D.shape
    return D.new_empty((B,)), D.new_empty((_native.score_elems(B, N, M),), dtype=torch.float32)


@torch.library.custom_op("softdtw_cuda::d_backward", mutates_args=(), device_types="cuda")
def d_backward(score: Tensor, grad_out: Tensor, B: int, N: int, M: int, gamma: float, bandwidth: float) -> Tensor:
    return _native.backward(score, grad_out, B, N, M, gamma, bandwidth)


@d_backward.register_fake
def _(score, grad_out, B, N, M, gamma, bandwidth):
    return score.new_empty((B, N, M), dtype=torch.float32)


def _d_setup(ctx, inputs, output):
    D, gamma, bandwidth = inputs
    ctx.save_for_backward(output[1])
    ctx.dims = tuple(D.shape)
    ctx.dtype = D.dtype
    ctx.gamma, ctx.bandwidth = gamma, bandwidth


def _d_backward(ctx, grad_out, _grad_score):
    (score,) = ctx.saved_tensors
    B, N, M = ctx.dims
    E = d_backward(score, grad_out, B, N, M, ctx.gamma, ctx.bandwidth)
    return E.to(ctx.dtype), None, None


d_forward.register_autograd(_d_backward, setup_context=_d_setup)
