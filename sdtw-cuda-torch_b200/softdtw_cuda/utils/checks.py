"""Input checks for the cost-matrix entry point (softdtw_cuda/utils/checks.py:6-15)."""
from __future__ import annotations

import torch

_FLOAT_DTYPES = (torch.float32, torch.float64, torch.float16, torch.bfloat16)


def check_D(D: torch.Tensor) -> None:
    """A cost matrix must be a 3-D floating tensor (B, N, M).

    Non-contiguous inputs are accepted; the launchers make them contiguous.
    """
    if not isinstance(D, torch.Tensor):
        raise TypeError("D must be a torch.Tensor")
    if D.dim() != 3:
        raise ValueError(f"D must have shape (B,N,M). Got {tuple(D.shape)}")
    if D.dtype not in _FLOAT_DTYPES:
        raise TypeError(f"Unsupported dtype {D.dtype}")
