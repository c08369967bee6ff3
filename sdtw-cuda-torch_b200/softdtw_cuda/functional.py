"""Functional form of the loss (softdtw_cuda/functional.py:7-25)."""
from __future__ import annotations

import torch

from .module import SoftDTW


def softdtw(
    x: torch.Tensor,
    y: torch.Tensor,
    *,
    gamma: float = 1.0,
    bandwidth: float | None = None,
    normalize: bool = False,
    dist: str = "sqeuclidean",
    fused: bool | None = None,
) -> torch.Tensor:
    """Soft-DTW between x (B,N,D) or (N,D) and y (B,M,D) or (M,D); returns (B,).

    fused: None picks the fused kernels when possible, True requires them,
    False always builds the cost matrix.
    """
    return SoftDTW(gamma=gamma, bandwidth=bandwidth, normalize=normalize, dist=dist, fused=fused)(x, y)
