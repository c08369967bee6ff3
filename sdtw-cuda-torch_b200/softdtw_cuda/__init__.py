"""softdtw_cuda -- Soft-DTW for PyTorch on NVIDIA B200 (sm_100a).

Drop-in for the public API of BGU-CS-VIL/sdtw-cuda-torch
(softdtw_cuda/__init__.py:1-5): the same four names, arguments and errors.
CUDA tensors run on the hand-written kernels of libsdtw_b200.so; CPU tensors run
on the library's host implementation.
"""
from .functional import softdtw
from .module import SoftDTW
from .barycenters import softdtw_barycenter, softdtw_barycenter_cpu

__all__ = ["softdtw", "SoftDTW", "softdtw_barycenter", "softdtw_barycenter_cpu"]
__version__ = "0.1.0"
