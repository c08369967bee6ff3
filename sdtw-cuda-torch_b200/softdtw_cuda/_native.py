"""ctypes binding of libsdtw_b200.so (the C ABI declared in include/sdtw_b200.h).

Every CUDA tensor operation of the package goes through this module.  There is
no fallback: if the library is missing or a call fails, a RuntimeError is
raised.  PyTorch supplies device memory (outputs and workspaces) and the
current CUDA stream; the kernels are the library's.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libsdtw_b200.so")

_lib = None
_lock = threading.Lock()

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Dbl = ctypes.c_double
_SZ = ctypes.c_size_t

_SIGS = {
    "sdtw_version": ([], ctypes.c_char_p),
    "sdtw_error_string": ([_I], ctypes.c_char_p),
    "sdtw_last_error_message": ([], ctypes.c_char_p),
    "sdtw_status": ([], _I),
    "sdtw_set_wait_timeout_ns": ([ctypes.c_ulonglong], None),
    "sdtw_debug_stall_stripe": ([_I], None),
    "sdtw_timing_enable": ([_I], None),
    "sdtw_timing_read": ([ctypes.c_char_p, _SZ, _P, _P, _I], _I),
    "sdtw_set_plan_override": ([_I, _I, _I], None),
    "sdtw_plan_info": ([_I, _I, _I, _P], _I),
    "sdtw_launch_count": ([], ctypes.c_ulonglong),
    "sdtw_score_elems": ([_I, _I, _I], _SZ),
    "sdtw_cost_elems": ([_I, _I, _I], _SZ),
    "sdtw_workspace_bytes": ([_I, _I, _I], _SZ),
    "sdtw_workspace_bytes_xy": ([_I, _I, _I, _I], _SZ),
    "sdtw_cost_sqeuclid_f32": ([_P, _P, _P, _I, _I, _I, _I, _I, _P], _I),
    "sdtw_forward_f32": ([_P, _P, _P, _I, _I, _I, _F, _F, _P, _SZ, _P], _I),
    "sdtw_backward_f32": ([_P, _P, _P, _I, _I, _I, _F, _F, _P, _SZ, _P], _I),
    "sdtw_forward_xy_f32": ([_P, _P, _P, _P, _I, _I, _I, _I, _F, _F, _P, _SZ, _P], _I),
    "sdtw_backward_xy_f32": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _F, _P, _SZ, _P], _I),
    "sdtw_forward_noalloc_f32": ([_P, _P, _P, _I, _I, _I, _F, _F, _P], _I),
    "sdtw_forward_sqeuclid_f32": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _F, _P, _SZ, _P], _I),
    "sdtw_backward_sqeuclid_f32": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _F, _P, _SZ, _P], _I),
    "sdtw_grad_sqeuclid_f32": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P], _I),
    "sdtw_workspace_bytes_norm": ([_I, _I, _I], _SZ),
    "sdtw_forward_xy_norm_f32": ([_P, _P, _P, _P, _I, _I, _I, _F, _F, _P, _SZ, _P], _I),
    "sdtw_backward_xy_norm_f32": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _F, _P, _SZ, _P], _I),
    "sdtw_forward_sqeuclid_norm_f32": ([_P, _P, _P, _P, _P, _I, _I, _I, _F, _F, _P, _SZ, _P], _I),
    "sdtw_backward_sqeuclid_norm_f32": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _F, _P, _SZ, _P], _I),
    "sdtw_score_to_R_f32": ([_P, _P, _I, _I, _I, _F, _P], _I),
    "sdtw_R_to_score_f32": ([_P, _P, _I, _I, _I, _F, _P], _I),
    "sdtw_forward_f64": ([_P, _P, _P, _I, _I, _I, _Dbl, _Dbl, _P], _I),
    "sdtw_backward_f64": ([_P, _P, _P, _P, _I, _I, _I, _Dbl, _Dbl, _P], _I),
    "sdtw_cost_sqeuclid_f64": ([_P, _P, _P, _I, _I, _I, _I, _P], _I),
    "sdtw_grad_sqeuclid_f64": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _P], _I),
    "sdtw_barycenter_workspace_bytes": ([_I, _I, _I, _I], _SZ),
    "sdtw_barycenter_grad_f32": ([_P, _P, _P, _P, _I, _I, _I, _I, _F, _P, _SZ, _P], _I),
    "sdtw_barycenter_adam_f32": ([_P, _P, _P, _P, _SZ, _P, _I, _P, _P, _P, _F, _F, _F, _F, _P], _I),
    "sdtw_barycenter_sync_bytes": ([_SZ, _I], _SZ),
    "sdtw_barycenter_sync_adam_f32": ([_P, _SZ, _P, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _F, _F, _F, _F, _P],
                                      _I),
    "sdtw_cpu_forward_f64": ([_P, _P, _P, _I, _I, _I, _Dbl, _Dbl], _I),
    "sdtw_cpu_backward_f64": ([_P, _P, _P, _I, _I, _I, _Dbl, _Dbl], _I),
}

# Every symbol the header declares (tests check the library exports them).
EXPORTED = tuple(_SIGS)


def lib():
    """Load the library once (RuntimeError if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"softdtw_cuda: native library {LIB_PATH} is missing; build it with "
                    "`python -m softdtw_cuda._build` (or __graft_entry__.build())")
            L = ctypes.CDLL(LIB_PATH)
            for name, (args, res) in _SIGS.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = res
            _lib = L
    return _lib


class NativeError(RuntimeError):
    pass


def launches() -> int:
    """Kernels the library has launched since it was loaded (its own counter)."""
    return int(lib().sdtw_launch_count())


# When a list, every op appends (name, start_event, end_event) recorded on the
# stream it launched on (used by bench.py for per-kernel timing).
profile_events = None


def _op_begin(device):
    if profile_events is None:
        return None
    ev = torch.cuda.Event(enable_timing=True)
    ev.record(torch.cuda.current_stream(device))
    return ev


def _op_end(name, device, ev0, n_kernels=None):
    if ev0 is not None:
        ev1 = torch.cuda.Event(enable_timing=True)
        ev1.record(torch.cuda.current_stream(device))
        profile_events.append((name, ev0, ev1))


def _check(rc: int, what: str) -> None:
    if rc != 0:
        L = lib()
        msg = L.sdtw_last_error_message().decode(errors="replace")
        kind = L.sdtw_error_string(rc).decode(errors="replace")
        raise NativeError(f"softdtw_cuda: {what} failed: {kind}: {msg}")


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


_SAME_DEVICE = contextlib.nullcontext()


def _on(device: torch.device):
    """The device's context for a library call: a no-op when it is already current."""
    if device.index is None or device.index == torch.cuda.current_device():
        return _SAME_DEVICE
    return torch.cuda.device(device)


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def status() -> int:
    """Read and clear the device wait status (0 = ok).  Synchronise first."""
    return int(lib().sdtw_status())


def check_status(device=None) -> None:
    """Synchronise ``device`` and raise if a device-side wait timed out."""
    if torch.cuda.is_available():
        torch.cuda.synchronize(device)
    s = status()
    if s != 0:
        raise NativeError(f"softdtw_cuda: device-side wait failed (status {s}): "
                          f"{lib().sdtw_last_error_message().decode(errors='replace')}")


def set_plan_override(warps_per_cta: int = 0, cluster_size: int = 0, rows_per_lane: int = 0) -> None:
    """Force the wavefront launch geometry (zeros restore the automatic plan).
    A forward and its backward must run under the same rows_per_lane."""
    lib().sdtw_set_plan_override(int(warps_per_cta), int(cluster_size), int(rows_per_lane))


def plan_info(B: int, N: int, M: int) -> dict:
    """Launch geometry the library chooses for a (B, N, M) problem on the
    current device (diagnostic)."""
    info = (ctypes.c_int * 6)()
    _check(lib().sdtw_plan_info(int(B), int(N), int(M), info), "plan_info")
    keys = ("rows_per_lane", "warps_per_cta", "cluster_size", "bands", "stripes", "clusters_fit")
    return dict(zip(keys, list(info)))


def set_wait_timeout(seconds: float) -> None:
    lib().sdtw_set_wait_timeout_ns(int(seconds * 1e9))


def debug_stall_stripe(stripe: int) -> None:
    lib().sdtw_debug_stall_stripe(int(stripe))


def timing_enable(on: bool = True) -> None:
    """Bracket every library kernel with CUDA events on its stream (clears totals)."""
    lib().sdtw_timing_enable(1 if on else 0)


def timing_read() -> dict:
    """{kernel name: (total ms, launches)} since timing_enable (synchronises the events)."""
    import numpy as np
    buf = ctypes.create_string_buffer(4096)
    ms = np.zeros(64, dtype=np.float64)
    cnt = np.zeros(64, dtype=np.int64)
    n = lib().sdtw_timing_read(buf, 4096, ms.ctypes.data_as(ctypes.c_void_p), cnt.ctypes.data_as(ctypes.c_void_p), 64)
    names = buf.value.decode().split(",") if n else []
    return {names[i]: (float(ms[i]), int(cnt[i])) for i in range(n)}


def version() -> str:
    return lib().sdtw_version().decode()


# ----------------------------------------------------------------------------- sizes
def score_elems(B: int, N: int, M: int) -> int:
    return int(lib().sdtw_score_elems(B, N, M))


def cost_elems(B: int, N: int, M: int) -> int:
    return int(lib().sdtw_cost_elems(B, N, M))


def workspace(B: int, N: int, M: int, device, dim: int | None = None) -> torch.Tensor:
    """Caller-owned scratch of the size the library asks for (torch allocations
    are 256-byte aligned, as the library requires)."""
    L = lib()
    n = L.sdtw_workspace_bytes(B, N, M) if dim is None else L.sdtw_workspace_bytes_xy(B, N, M, dim)
    return torch.empty(max(int(n), 256), dtype=torch.uint8, device=device)


def _f32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype is torch.float32 and t.is_contiguous():
        return t.detach()
    return t.detach().to(dtype=torch.float32).contiguous()


# ----------------------------------------------------------------------------- CUDA ops
def barycenter_workspace(B: int, N: int, M: int, dim: int, device) -> torch.Tensor:
    n = lib().sdtw_barycenter_workspace_bytes(B, N, M, dim)
    return torch.empty(max(int(n), 256), dtype=torch.uint8, device=device)


def barycenter_grad(bary: torch.Tensor, X: torch.Tensor, w: torch.Tensor, grad_loss: torch.Tensor, gamma: float,
                    ws: torch.Tensor) -> None:
    """grad_loss (N*D + 1,) <- [sum_b w_b dSoftDTW(bary, X_b)/dbary | sum_b w_b SoftDTW(bary, X_b)].
    All operands contiguous float32 on one device (not copied: the call can
    be captured in a CUDA graph)."""
    B, M, dim = X.shape
    N = bary.shape[0]
    for t in (bary, X, w, grad_loss):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.device != X.device:
            raise ValueError("barycenter_grad: operands must be contiguous float32 tensors on one device")
    if bary.shape != (N, dim) or w.shape != (B,) or grad_loss.numel() != N * dim + 1:
        raise ValueError("barycenter_grad: shape mismatch")
    with _on(X.device):
        rc = lib().sdtw_barycenter_grad_f32(_ptr(bary), _ptr(X), _ptr(w), _ptr(grad_loss), B, N, M, dim,
                                            float(gamma), _ptr(ws), ws.numel(), _stream(X.device))
    _check(rc, "barycenter gradient")


def barycenter_adam(bary, exp_avg, exp_avg_sq, grad_loss, lr_table, step, loss_hist, bary_hist,
                    beta1=0.9, beta2=0.999, eps=1e-8, max_norm=1.0) -> None:
    """Clip grad_loss[:n] to max_norm, one Adam step on bary with lr_table[step],
    record the loss and the new bary at index step, step += 1 (all on the device)."""
    n = bary.numel()
    if step.dtype != torch.int32:
        raise ValueError("barycenter_adam: step must be an int32 tensor")
    with _on(bary.device):
        rc = lib().sdtw_barycenter_adam_f32(_ptr(bary), _ptr(exp_avg), _ptr(exp_avg_sq), _ptr(grad_loss), n,
                                            _ptr(lr_table), lr_table.numel(), _ptr(step), _ptr(loss_hist),
                                            _ptr(bary_hist), float(beta1), float(beta2), float(eps), float(max_norm),
                                            _stream(bary.device))
    _check(rc, "barycenter Adam step")


def barycenter_sync_bytes(n: int, world: int) -> int:
    return int(lib().sdtw_barycenter_sync_bytes(n, world))


def barycenter_sync_adam(grad_loss, peers, world, rank, epoch, bary, exp_avg, exp_avg_sq, lr_table, step, loss_hist,
                         bary_hist, beta1=0.9, beta2=0.999, eps=1e-8, max_norm=1.0) -> None:
    """Sum grad_loss (n + 1,) over the ranks through the exchange buffers whose
    addresses `peers` (int64 device tensor, one per rank) holds, then the Adam
    step of barycenter_adam.  `epoch`: int64 device counter (zero at first)."""
    n = bary.numel()
    if step.dtype != torch.int32 or epoch.dtype != torch.int64 or peers.dtype != torch.int64:
        raise ValueError("barycenter_sync_adam: step int32, epoch and peers int64 tensors")
    with _on(bary.device):
        rc = lib().sdtw_barycenter_sync_adam_f32(_ptr(grad_loss), n, _ptr(peers), int(world), int(rank), _ptr(epoch),
                                                 _ptr(bary), _ptr(exp_avg), _ptr(exp_avg_sq), _ptr(lr_table),
                                                 lr_table.numel(), _ptr(step), _ptr(loss_hist), _ptr(bary_hist),
                                                 float(beta1), float(beta2), float(eps), float(max_norm),
                                                 _stream(bary.device))
    _check(rc, "barycenter exchange and Adam step")


def cost_sqeuclid(x: torch.Tensor, y: torch.Tensor, direct: bool = False) -> torch.Tensor:
    x = _f32(x)
    y = _f32(y)
    B, N, dim = x.shape
    M = y.shape[1]
    D = torch.empty((B, N, M), dtype=torch.float32, device=x.device)
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_cost_sqeuclid_f32(_ptr(x), _ptr(y), _ptr(D), B, N, M, dim, int(direct), _stream(x.device))
    _check(rc, "cost")
    _op_end("cost", x.device, ev)
    return D


def forward(D: torch.Tensor, gamma: float, bandwidth: float):
    """(out (B,), score) for a CUDA cost tensor D (B,N,M)."""
    D = _f32(D)
    B, N, M = D.shape
    score = torch.empty(score_elems(B, N, M), dtype=torch.float32, device=D.device)
    out = torch.empty(B, dtype=torch.float32, device=D.device)
    ws = workspace(B, N, M, D.device)
    ev = _op_begin(D.device)
    with _on(D.device):
        rc = lib().sdtw_forward_f32(_ptr(D), _ptr(score), _ptr(out), B, N, M, float(gamma), float(bandwidth),
                                    _ptr(ws), ws.numel(), _stream(D.device))
    _check(rc, "forward")
    _op_end("forward", D.device, ev)
    return out, score


def backward(score: torch.Tensor, grad_out: torch.Tensor | None, B: int, N: int, M: int, gamma: float,
             bandwidth: float) -> torch.Tensor:
    """E (B,N,M) = grad_out[b] * dR[N,M]/dD."""
    dev = score.device
    E = torch.empty((B, N, M), dtype=torch.float32, device=dev)
    g = None if grad_out is None else _f32(grad_out.reshape(-1))
    ws = workspace(B, N, M, dev)
    ev = _op_begin(dev)
    with _on(dev):
        rc = lib().sdtw_backward_f32(_ptr(score), _ptr(g), _ptr(E), B, N, M, float(gamma), float(bandwidth),
                                     _ptr(ws), ws.numel(), _stream(dev))
    _check(rc, "backward")
    _op_end("backward", dev, ev)
    return E


def forward_xy(x: torch.Tensor, y: torch.Tensor, gamma: float, bandwidth: float):
    x = _f32(x)
    y = _f32(y)
    B, N, dim = x.shape
    M = y.shape[1]
    score = torch.empty(score_elems(B, N, M), dtype=torch.float32, device=x.device)
    out = torch.empty(B, dtype=torch.float32, device=x.device)
    ws = workspace(B, N, M, x.device, dim)
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_forward_xy_f32(_ptr(x), _ptr(y), _ptr(score), _ptr(out), B, N, M, dim, float(gamma),
                                       float(bandwidth), _ptr(ws), ws.numel(), _stream(x.device))
    _check(rc, "fused forward")
    _op_end("forward_xy", x.device, ev)
    return out, score


def backward_xy(x: torch.Tensor, y: torch.Tensor, score: torch.Tensor, grad_out: torch.Tensor | None,
                gamma: float, bandwidth: float, need_x: bool = True, need_y: bool = True):
    x = _f32(x)
    y = _f32(y)
    B, N, dim = x.shape
    M = y.shape[1]
    gx = torch.empty_like(x) if need_x else None
    gy = torch.empty_like(y) if need_y else None
    g = None if grad_out is None else _f32(grad_out.reshape(-1))
    ws = workspace(B, N, M, x.device, dim)
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_backward_xy_f32(_ptr(x), _ptr(y), _ptr(score), _ptr(g), _ptr(gx), _ptr(gy), B, N, M, dim,
                                        float(gamma), float(bandwidth), _ptr(ws), ws.numel(), _stream(x.device))
    _check(rc, "fused backward")
    _op_end("backward_xy", x.device, ev, 2 + int(need_x) + int(need_y))
    return gx, gy


def forward_sqeuclid(x: torch.Tensor, y: torch.Tensor, gamma: float, bandwidth: float):
    """Unfused path: (out, score, cost) with the clamped expanded cost kept for the backward."""
    x = _f32(x)
    y = _f32(y)
    B, N, dim = x.shape
    M = y.shape[1]
    score = torch.empty(score_elems(B, N, M), dtype=torch.float32, device=x.device)
    cost = torch.empty(cost_elems(B, N, M), dtype=torch.float32, device=x.device)
    out = torch.empty(B, dtype=torch.float32, device=x.device)
    ws = workspace(B, N, M, x.device)
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_forward_sqeuclid_f32(_ptr(x), _ptr(y), _ptr(score), _ptr(cost), _ptr(out), B, N, M, dim,
                                             float(gamma), float(bandwidth), _ptr(ws), ws.numel(), _stream(x.device))
    _check(rc, "unfused forward")
    _op_end("forward_sqeuclid", x.device, ev)
    return out, score, cost


def backward_sqeuclid(x: torch.Tensor, y: torch.Tensor, score: torch.Tensor, cost: torch.Tensor,
                      grad_out: torch.Tensor | None, gamma: float, bandwidth: float, need_x: bool = True,
                      need_y: bool = True):
    x = _f32(x)
    y = _f32(y)
    B, N, dim = x.shape
    M = y.shape[1]
    gx = torch.empty_like(x) if need_x else None
    gy = torch.empty_like(y) if need_y else None
    g = None if grad_out is None else _f32(grad_out.reshape(-1))
    ws = workspace(B, N, M, x.device, dim)
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_backward_sqeuclid_f32(_ptr(x), _ptr(y), _ptr(score), _ptr(cost), _ptr(g), _ptr(gx), _ptr(gy),
                                              B, N, M, dim, float(gamma), float(bandwidth), _ptr(ws), ws.numel(),
                                              _stream(x.device))
    _check(rc, "unfused backward")
    _op_end("backward_sqeuclid", x.device, ev, 2 + int(need_x) + int(need_y))
    return gx, gy


# ----------------------------------------------------------------------------- normalize=True
# The 3B problems (x_b, y_b), (x_b, x_b), (y_b, y_b) read x and y in place
# (softdtw_cuda/module.py:99-111 of the reference concatenates copies).
def _norm_pair(x: torch.Tensor, y: torch.Tensor):
    if x.dim() != 3 or x.shape != y.shape or not (x.is_cuda and y.is_cuda) or x.device != y.device:
        raise ValueError(f"normalize: expected CUDA x, y of one shape (B,N,D); got {tuple(x.shape)}, {tuple(y.shape)}")
    return _f32(x), _f32(y)


def _norm_ws(B: int, N: int, dim: int, device) -> torch.Tensor:
    n = lib().sdtw_workspace_bytes_norm(B, N, dim)
    return torch.empty(max(int(n), 256), dtype=torch.uint8, device=device)


def forward_xy_norm(x: torch.Tensor, y: torch.Tensor, gamma: float, bandwidth: float):
    """Fused forward of the normalized triple: (out (3B,) [xy | xx | yy], score)."""
    x, y = _norm_pair(x, y)
    B, N, dim = x.shape
    score = torch.empty(score_elems(3 * B, N, N), dtype=torch.float32, device=x.device)
    out = torch.empty(3 * B, dtype=torch.float32, device=x.device)
    ws = workspace(3 * B, N, N, x.device, dim)
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_forward_xy_norm_f32(_ptr(x), _ptr(y), _ptr(score), _ptr(out), B, N, dim, float(gamma),
                                            float(bandwidth), _ptr(ws), ws.numel(), _stream(x.device))
    _check(rc, "fused normalized forward")
    _op_end("forward_xy", x.device, ev)
    return out, score


def backward_xy_norm(x: torch.Tensor, y: torch.Tensor, score: torch.Tensor, grad_out: torch.Tensor | None,
                     gamma: float, bandwidth: float):
    """grad_x, grad_y of sum_p grad_out[p] * out[p] over the normalized triple."""
    x, y = _norm_pair(x, y)
    B, N, dim = x.shape
    gx = torch.empty_like(x)
    gy = torch.empty_like(y)
    g = None if grad_out is None else _f32(grad_out.reshape(-1))
    if g is not None and g.numel() != 3 * B:
        raise ValueError(f"normalize: expected {3 * B} upstream gradients, got {g.numel()}")
    ws = _norm_ws(B, N, dim, x.device)
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_backward_xy_norm_f32(_ptr(x), _ptr(y), _ptr(score), _ptr(g), _ptr(gx), _ptr(gy), B, N, dim,
                                             float(gamma), float(bandwidth), _ptr(ws), ws.numel(), _stream(x.device))
    _check(rc, "fused normalized backward")
    _op_end("backward_xy", x.device, ev)
    return gx, gy


def forward_sqeuclid_norm(x: torch.Tensor, y: torch.Tensor, gamma: float, bandwidth: float):
    """Unfused forward of the normalized triple: (out (3B,), score, cost)."""
    x, y = _norm_pair(x, y)
    B, N, dim = x.shape
    score = torch.empty(score_elems(3 * B, N, N), dtype=torch.float32, device=x.device)
    cost = torch.empty(cost_elems(3 * B, N, N), dtype=torch.float32, device=x.device)
    out = torch.empty(3 * B, dtype=torch.float32, device=x.device)
    ws = workspace(3 * B, N, N, x.device)
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_forward_sqeuclid_norm_f32(_ptr(x), _ptr(y), _ptr(score), _ptr(cost), _ptr(out), B, N, dim,
                                                  float(gamma), float(bandwidth), _ptr(ws), ws.numel(),
                                                  _stream(x.device))
    _check(rc, "unfused normalized forward")
    _op_end("forward_sqeuclid", x.device, ev)
    return out, score, cost


def backward_sqeuclid_norm(x: torch.Tensor, y: torch.Tensor, score: torch.Tensor, cost: torch.Tensor,
                           grad_out: torch.Tensor | None, gamma: float, bandwidth: float):
    x, y = _norm_pair(x, y)
    B, N, dim = x.shape
    gx = torch.empty_like(x)
    gy = torch.empty_like(y)
    g = None if grad_out is None else _f32(grad_out.reshape(-1))
    if g is not None and g.numel() != 3 * B:
        raise ValueError(f"normalize: expected {3 * B} upstream gradients, got {g.numel()}")
    ws = _norm_ws(B, N, dim, x.device)
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_backward_sqeuclid_norm_f32(_ptr(x), _ptr(y), _ptr(score), _ptr(cost), _ptr(g), _ptr(gx),
                                                   _ptr(gy), B, N, dim, float(gamma), float(bandwidth), _ptr(ws),
                                                   ws.numel(), _stream(x.device))
    _check(rc, "unfused normalized backward")
    _op_end("backward_sqeuclid", x.device, ev)
    return gx, gy


def grad_sqeuclid(G: torch.Tensor, D_mask: torch.Tensor | None, x: torch.Tensor, y: torch.Tensor,
                  need_x: bool = True, need_y: bool = True):
    G = _f32(G)
    x = _f32(x)
    y = _f32(y)
    Dm = None if D_mask is None else _f32(D_mask)
    B, N, dim = x.shape
    M = y.shape[1]
    gx = torch.empty_like(x) if need_x else None
    gy = torch.empty_like(y) if need_y else None
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_grad_sqeuclid_f32(_ptr(G), _ptr(Dm), _ptr(x), _ptr(y), _ptr(gx), _ptr(gy), B, N, M, dim,
                                          _stream(x.device))
    _check(rc, "cost gradient")
    _op_end("grad_sqeuclid", x.device, ev, int(need_x) + int(need_y))
    return gx, gy


def score_to_R(score: torch.Tensor, B: int, N: int, M: int, gamma: float) -> torch.Tensor:
    R = torch.empty((B, N + 2, M + 2), dtype=torch.float32, device=score.device)
    with _on(score.device):
        rc = lib().sdtw_score_to_R_f32(_ptr(score), _ptr(R), B, N, M, float(gamma), _stream(score.device))
    _check(rc, "score_to_R")
    _op_end("score_to_R", score.device, None)
    return R


def R_to_score(R: torch.Tensor, gamma: float) -> torch.Tensor:
    R = _f32(R)
    B, N2, M2 = R.shape
    N, M = N2 - 2, M2 - 2
    score = torch.empty(score_elems(B, N, M), dtype=torch.float32, device=R.device)
    with _on(R.device):
        rc = lib().sdtw_R_to_score_f32(_ptr(R), _ptr(score), B, N, M, float(gamma), _stream(R.device))
    _check(rc, "R_to_score")
    _op_end("R_to_score", R.device, None)
    return score


# ----------------------------------------------------------------------------- CUDA float64 ops
def _f64(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(dtype=torch.float64).contiguous()


def forward_f64(D: torch.Tensor, gamma: float, bandwidth: float):
    """(out (B,), R (B,N+2,M+2)) in float64 for a CUDA float64 cost tensor."""
    D = _f64(D)
    B, N, M = D.shape
    R = torch.empty((B, N + 2, M + 2), dtype=torch.float64, device=D.device)
    out = torch.empty(B, dtype=torch.float64, device=D.device)
    ev = _op_begin(D.device)
    with _on(D.device):
        rc = lib().sdtw_forward_f64(_ptr(D), _ptr(R), _ptr(out), B, N, M, float(gamma), float(bandwidth),
                                    _stream(D.device))
    _check(rc, "float64 forward")
    _op_end("forward_f64", D.device, ev)
    return out, R


def backward_f64(D: torch.Tensor, R: torch.Tensor, grad_out: torch.Tensor | None, gamma: float,
                 bandwidth: float) -> torch.Tensor:
    """E (B,N,M) = grad_out[b] * dR[N,M]/dD in float64 on the GPU."""
    D = _f64(D)
    B, N, M = D.shape
    E = torch.empty((B, N, M), dtype=torch.float64, device=D.device)
    g = None if grad_out is None else grad_out.detach().reshape(-1).to(device=D.device, dtype=torch.float64).contiguous()
    ev = _op_begin(D.device)
    with _on(D.device):
        rc = lib().sdtw_backward_f64(_ptr(D), _ptr(R), _ptr(g), _ptr(E), B, N, M, float(gamma), float(bandwidth),
                                     _stream(D.device))
    _check(rc, "float64 backward")
    _op_end("backward_f64", D.device, ev)
    return E


def cost_sqeuclid_f64(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """D = sum_k (x_ik - y_jk)^2 in float64 on the GPU (the fused cost's direct form)."""
    x = _f64(x)
    y = _f64(y)
    B, N, dim = x.shape
    M = y.shape[1]
    D = torch.empty((B, N, M), dtype=torch.float64, device=x.device)
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_cost_sqeuclid_f64(_ptr(x), _ptr(y), _ptr(D), B, N, M, dim, _stream(x.device))
    _check(rc, "float64 cost")
    _op_end("cost_f64", x.device, ev)
    return D


def grad_sqeuclid_f64(G: torch.Tensor, x: torch.Tensor, y: torch.Tensor, need_x: bool = True,
                      need_y: bool = True):
    """grad_x = 2 (x rowsum(G) - G y), grad_y = 2 (y colsum(G) - G^T x) in float64 on the GPU."""
    G = _f64(G)
    x = _f64(x)
    y = _f64(y)
    B, N, dim = x.shape
    M = y.shape[1]
    gx = torch.empty_like(x) if need_x else None
    gy = torch.empty_like(y) if need_y else None
    ev = _op_begin(x.device)
    with _on(x.device):
        rc = lib().sdtw_grad_sqeuclid_f64(_ptr(G), _ptr(x), _ptr(y), _ptr(gx), _ptr(gy), B, N, M, dim,
                                          _stream(x.device))
    _check(rc, "float64 chain rule")
    _op_end("grad_f64", x.device, ev)
    return gx, gy


# ----------------------------------------------------------------------------- CPU ops
def cpu_forward(D: torch.Tensor, gamma: float, bandwidth: float):
    """(out, R) in float64 for a CPU cost tensor; R uses the reference layout."""
    Dd = D.detach().to(dtype=torch.float64).contiguous()
    B, N, M = Dd.shape
    R = torch.empty((B, N + 2, M + 2), dtype=torch.float64)
    out = torch.empty(B, dtype=torch.float64)
    rc = lib().sdtw_cpu_forward_f64(_ptr(Dd), _ptr(R), _ptr(out), B, N, M, float(gamma), float(bandwidth))
    _check(rc, "cpu forward")
    return out, R


def cpu_backward(R: torch.Tensor, grad_out: torch.Tensor | None, gamma: float, bandwidth: float) -> torch.Tensor:
    Rd = R.detach().to(dtype=torch.float64).contiguous()
    B, N2, M2 = Rd.shape
    N, M = N2 - 2, M2 - 2
    E = torch.empty((B, N, M), dtype=torch.float64)
    g = None if grad_out is None else grad_out.detach().reshape(-1).to(dtype=torch.float64).contiguous()
    rc = lib().sdtw_cpu_backward_f64(_ptr(Rd), _ptr(g), _ptr(E), B, N, M, float(gamma), float(bandwidth))
    _check(rc, "cpu backward")
    return E
