"""CPU parity oracle for the Soft-DTW hot path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference`` arm) may import this module, and
only as the checker or the timed CPU baseline.  The product package
``softdtw_cuda`` never imports it.

The dynamic programme itself lives in ``sdtw_oracle.c`` (built into
``liboracle_sdtw.so`` by ``oracle/Makefile``); this module adds the numpy
pieces of the reference pipeline around it:

* ``sqeuclid``            softdtw_cuda/distances.py:6-28  (expanded form, clamp >= 0)
* ``cost_direct``         softdtw_cuda/cuda/kernels.py:27-31 (fused-mode cost)
* ``forward``/``backward`` softdtw_cuda/cuda/launcher.py:356-368
* ``loss_and_grads``      softdtw_cuda/module.py:66-118, autograd.py:11-48,
                          autograd_xy.py:12-51 and the autograd of distances.py
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_sdtw.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile liboracle_sdtw.so with oracle/Makefile (gcc + OpenMP)."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I = ctypes.c_int
        Dd = ctypes.c_double
        L.oracle_forward_f32.argtypes = [P, I, I, I, Dd, Dd, P, P]
        L.oracle_forward_f64.argtypes = [P, I, I, I, Dd, Dd, P]
        L.oracle_backward_f32.argtypes = [P, P, I, I, I, Dd, Dd, P]
        L.oracle_backward_f64.argtypes = [P, P, I, I, I, Dd, Dd, P]
        L.oracle_cost_direct_f32.argtypes = [P, P, I, I, I, I, P]
        L.oracle_num_threads.restype = I
        L.oracle_set_num_threads.argtypes = [I]
        L.oracle_set_num_threads.restype = None
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _bw(bandwidth) -> float:
    # autograd.py:19-23: None or <= 0 means disabled (-1).
    if bandwidth is None:
        return -1.0
    bw = float(bandwidth)
    return -1.0 if bw <= 0 else bw


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


def forward(D: np.ndarray, gamma: float, bandwidth=None):
    """launcher.py:356-361.  Returns (out (B,), R (B,N+2,M+2)) in D's dtype,
    plus the float64 table the reference keeps internally."""
    D = np.ascontiguousarray(D)
    B, N, M = D.shape
    R64 = np.empty((B, N + 2, M + 2), dtype=np.float64)
    if D.dtype == np.float32:
        R32 = np.empty((B, N + 2, M + 2), dtype=np.float32)
        lib().oracle_forward_f32(_ptr(D), B, N, M, float(gamma), _bw(bandwidth), _ptr(R64), _ptr(R32))
        R = R32
    elif D.dtype == np.float64:
        lib().oracle_forward_f64(_ptr(D), B, N, M, float(gamma), _bw(bandwidth), _ptr(R64))
        R = R64
    else:
        raise TypeError(f"oracle supports float32/float64, got {D.dtype}")
    return R[:, -2, -2].copy(), R, R64


def backward(D: np.ndarray, R: np.ndarray, gamma: float, bandwidth=None) -> np.ndarray:
    """launcher.py:364-368 (+ :327-353).  Returns E (B,N,M) in D's dtype."""
    D = np.ascontiguousarray(D)
    R = np.ascontiguousarray(R)
    B, N, M = D.shape
    E = np.empty((B, N, M), dtype=D.dtype)
    if D.dtype == np.float32:
        lib().oracle_backward_f32(_ptr(D), _ptr(R.astype(np.float32)), B, N, M, float(gamma),
                                  _bw(bandwidth), _ptr(E))
    else:
        lib().oracle_backward_f64(_ptr(D), _ptr(R.astype(np.float64)), B, N, M, float(gamma),
                                  _bw(bandwidth), _ptr(E))
    return E


def sqeuclid(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    """distances.py:6-28: ||x||^2 + ||y||^2 - 2 x y^T, clamped at 0, in x's dtype.
    Returns (D, pre) where pre is the unclamped value (for the clamp mask)."""
    x2 = (x * x).sum(-1)
    y2 = (y * y).sum(-1)
    xy = np.matmul(x, np.swapaxes(y, 1, 2))
    pre = x2[:, :, None] + y2[:, None, :] - x.dtype.type(2.0) * xy
    return np.maximum(pre, x.dtype.type(0.0)), pre


def cost_direct(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    """kernels.py:27-31: sum_k (x - y)^2 accumulated in double (float32 inputs)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.ascontiguousarray(y, dtype=np.float32)
    B, N, Dm = x.shape
    M = y.shape[1]
    D = np.empty((B, N, M), dtype=np.float64)
    lib().oracle_cost_direct_f32(_ptr(x), _ptr(y), B, N, M, Dm, _ptr(D))
    return D


def _chain_xy(G: np.ndarray, x: np.ndarray, y: np.ndarray, mask=None):
    """Gradient of sum_ij G_ij * ||x_i - y_j||^2 with respect to x and y
    (autograd_xy.py:41-49; the unfused path reaches the same expression through
    torch autograd of distances.py:20-28, with the clamp mask)."""
    if mask is not None:
        G = G * mask
    gx = 2.0 * (x * G.sum(2)[:, :, None] - np.matmul(G, y))
    gy = 2.0 * (y * G.sum(1)[:, :, None] - np.matmul(np.swapaxes(G, 1, 2), x))
    return gx, gy


def loss_and_grads(x, y, *, gamma=1.0, bandwidth=None, normalize=False, fused=False,
                   grad_out=None, precision="reference"):
    """Forward + backward of SoftDTW(x, y) as the reference computes it on CPU.

    precision="reference": float32 pipeline with the reference's dtype rules.
    precision="float64":   the same algorithm run on float64 copies (used as
                           the 'truth' the float32 results are measured against).
    fused=True uses the direct-difference cost of kernels.py:27-31 (the
    reference has no CPU fused mode; its CUDA fused kernels compute this cost).

    Returns (out (B,), grad_x, grad_y) where the grads are of sum(grad_out*out)
    (grad_out defaults to ones, i.e. loss = out.sum()).
    """
    x = np.asarray(x)
    y = np.asarray(y)
    if x.ndim == 2:
        x = x[None]
    if y.ndim == 2:
        y = y[None]
    dt = np.float64 if precision == "float64" else np.float32
    x = x.astype(dt)
    y = y.astype(dt)
    B = x.shape[0]
    if normalize:
        xc = np.concatenate([x, x, y], 0)
        yc = np.concatenate([y, x, y], 0)
    else:
        xc, yc = x, y
    if fused:
        Dc = cost_direct(xc.astype(np.float32), yc.astype(np.float32))
        D = Dc.astype(dt)
        mask = None
    else:
        D, pre = sqeuclid(xc, yc)
        mask = (pre >= 0).astype(dt)
    out, R, _ = forward(D, gamma, bandwidth)
    E = backward(D, R, gamma, bandwidth)
    if grad_out is None:
        g = np.ones(B, dtype=dt)
    else:
        g = np.asarray(grad_out, dtype=dt).reshape(B)
    if normalize:
        gc = np.concatenate([g, -0.5 * g, -0.5 * g]).astype(dt)
    else:
        gc = g
    G = E * gc[:, None, None]
    gx, gy = _chain_xy(G, xc, yc, mask)
    if normalize:
        oxy, oxx, oyy = out[:B], out[B:2 * B], out[2 * B:]
        res = oxy - 0.5 * (oxx + oyy)
        gx_t = gx[:B] + gx[B:2 * B] + gy[B:2 * B]
        gy_t = gy[:B] + gx[2 * B:] + gy[2 * B:]
        return res, gx_t, gy_t
    return out, gx, gy
