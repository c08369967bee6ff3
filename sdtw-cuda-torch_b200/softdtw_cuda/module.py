"""``SoftDTW`` loss module (softdtw_cuda/module.py:12-118).

Same constructor, dispatch policy, validation order and error messages as the
reference:

* ``fused=None`` uses the fused x/y kernels when both tensors are on the same
  CUDA device and ``dist`` is squared Euclidean; ``fused=True`` requires that;
  ``fused=False`` always builds the cost matrix.
* ``normalize=True`` returns SoftDTW(x,y) - (SoftDTW(x,x) + SoftDTW(y,y)) / 2,
  evaluated as one batch of 3B problems.  On CUDA float tensors the library
  reads x and y in place for the three pairs (no concatenated copies); other
  inputs (float64, CPU, other costs, torch.compile tracing) take the
  reference's concatenation.
"""
from __future__ import annotations

import math

import torch
from torch import nn

from . import ops  # noqa: F401  (registers torch.ops.softdtw_cuda.*)
from .autograd import SoftDTWAutograd, SoftDTWSqEuclidAutograd, SoftDTWSqEuclidNormAutograd, _normalize_bandwidth
from .autograd_xy import SoftDTWXYAutograd, SoftDTWXYNormAutograd
from .distances import _KERNEL_DTYPES, _SQEUCLID_NAMES, pairwise_distance


class SoftDTW(nn.Module):
    """Soft-DTW between batches of sequences x (B,N,D) and y (B,M,D); returns (B,).

    gamma      smoothing (> 0, finite)
    bandwidth  Sakoe-Chiba band half-width; None or <= 0 disables it
    normalize  subtract half of the self-similarities (requires N == M)
    dist       cost; only squared Euclidean ("sqeuclidean") is supported
    fused      None = auto, True = require the fused kernels, False = never
    """

    def __init__(
        self,
        *,
        gamma: float = 1.0,
        bandwidth: float | None = None,
        normalize: bool = False,
        dist: str = "sqeuclidean",
        fused: bool | None = None,
    ):
        super().__init__()
        g = float(gamma)
        if g <= 0:
            raise ValueError(f"gamma must be > 0, got {g}")
        if not math.isfinite(g):
            raise ValueError(f"gamma must be finite, got {g}")
        self.gamma = g
        if bandwidth is None or float(bandwidth) <= 0:
            self.bandwidth = None
        else:
            self.bandwidth = float(bandwidth)
        self.normalize = bool(normalize)
        self.dist = str(dist)
        self.fused = fused

    def _use_fused(self, x: torch.Tensor, y: torch.Tensor) -> bool:
        possible = (self.dist.lower() in _SQEUCLID_NAMES and x.is_cuda and y.is_cuda
                    and x.device == y.device)
        if self.fused is True and not possible:
            raise ValueError("fused=True requires CUDA tensors and dist='sqeuclidean'.")
        if self.fused is False:
            return False
        return possible

    def forward(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        if x.dim() == 2:
            x = x.unsqueeze(0)
        if y.dim() == 2:
            y = y.unsqueeze(0)
        if x.dim() != 3 or y.dim() != 3:
            raise ValueError(
                f"Expected x,y to have shape (B,N,D) and (B,M,D) (or unbatched (N,D)). "
                f"Got x={tuple(x.shape)}, y={tuple(y.shape)}")
        if self.normalize and x.shape[1] != y.shape[1]:
            raise ValueError(
                f"normalize=True currently requires equal sequence lengths (N==M) because it uses the "
                f"concatenation trick. Got N={x.shape[1]}, M={y.shape[1]}.")
        bx, _, dx = x.shape
        by, _, dy = y.shape
        if dx != dy:
            raise ValueError(f"Feature dims must match. Got x.shape[-1]={dx}, y.shape[-1]={dy}")
        if bx != by:
            raise ValueError(f"Batch sizes must match. Got x.shape[0]={bx}, y.shape[0]={by}")
        if x.shape[1] == 0 or y.shape[1] == 0:
            raise ValueError(f"Sequence lengths must be > 0. Got N={x.shape[1]}, M={y.shape[1]}.")

        use_fused = self._use_fused(x, y)
        if self.normalize:
            if self._kernel_pair(x, y) and not torch.compiler.is_compiling():
                fn = SoftDTWXYNormAutograd if use_fused else SoftDTWSqEuclidNormAutograd
                out = fn.apply(x, y, self.gamma, self.bandwidth)
            else:
                xs = torch.cat([x, x, y], dim=0)
                ys = torch.cat([y, x, y], dim=0)
                out = self._pairs(xs, ys, use_fused)
            o_xy, o_xx, o_yy = out.split(bx, dim=0)
            return o_xy - 0.5 * (o_xx + o_yy)
        return self._pairs(x, y, use_fused)

    def _kernel_pair(self, x: torch.Tensor, y: torch.Tensor) -> bool:
        # Squared Euclidean on CUDA tensors of one device and a float32 (or
        # bf16/fp16, computed in float32) dtype: the library's x/y kernels.
        return (self.dist.lower() in _SQEUCLID_NAMES and x.is_cuda and y.is_cuda and x.device == y.device
                and x.dtype in _KERNEL_DTYPES and y.dtype == x.dtype)

    def _pairs(self, x: torch.Tensor, y: torch.Tensor, use_fused: bool) -> torch.Tensor:
        if (torch.compiler.is_compiling() and self.dist.lower() in _SQEUCLID_NAMES and x.is_cuda and y.is_cuda
                and x.device == y.device and x.dtype in _KERNEL_DTYPES and y.dtype == x.dtype):
            # Under torch.compile: the same library calls as registered custom
            # operators (softdtw_cuda/ops.py), traceable without a graph break.
            if x.dim() != 3 or y.dim() != 3 or x.shape[0] != y.shape[0] or x.shape[2] != y.shape[2]:
                raise ValueError(f"Batch/features mismatch: {tuple(x.shape)} vs {tuple(y.shape)}")
            bw = _normalize_bandwidth(self.bandwidth)
            op = torch.ops.softdtw_cuda.xy_forward if use_fused else torch.ops.softdtw_cuda.sq_forward
            return op(x, y, float(self.gamma), bw)[0]
        if use_fused:
            return SoftDTWXYAutograd.apply(x, y, self.gamma, self.bandwidth)
        if self._kernel_pair(x, y):
            # Unfused: explicit cost matrix (kept by the library for the backward).
            return SoftDTWSqEuclidAutograd.apply(x, y, self.gamma, self.bandwidth)
        D = pairwise_distance(x, y, dist=self.dist)
        return SoftDTWAutograd.apply(D, self.gamma, self.bandwidth)
