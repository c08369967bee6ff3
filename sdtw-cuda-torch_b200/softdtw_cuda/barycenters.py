"""Soft-DTW barycenters (softdtw_cuda/barycenters.py:17-229).

The barycenter b (N,D) minimises sum_i w_i SoftDTW(b, X_i) by Adam with
gradient-norm clipping at 1.0 and cosine learning-rate annealing to lr/10;
optional early stopping on absolute loss improvement after half of max_iter
(the method of Cuturi & Blondel, ICML 2017).  Behaviour, defaults and
progress messages follow the reference.  The multi-GPU version is
``softdtw_cuda.distributed.sharded_barycenter``.

On CUDA the loop runs as one CUDA graph of one iteration, replayed
(barycenters.py:114-158 of the reference is a host loop with a device sync per
step): Soft-DTW forward and backward, the weighted loss, gradient clipping, an
Adam step with the learning rate read from a precomputed cosine-annealing table
indexed by a device iteration counter, and copies of the loss and of the
barycenter into per-iteration history buffers.  For float32 sequences and the
fused cost the iteration is the library's: the wavefronts read the one
barycenter for every sequence, the gradient and the loss are reduced over the
sequences on the device, and clipping, Adam and the histories are one kernel
(``_native.barycenter_grad`` / ``_native.barycenter_adam``).  The host reads
the loss history back asynchronously every few replays, applies the early-stop
rule to it, and returns the barycenter of the stopping iteration from the
history, so the result is the one the step-by-step loop returns.

The captured graph is kept (a few per process, keyed by the sequences'
address and shape and by gamma, lr, max_iter and the fused flag), so a second
call with the same configuration only resets the state and replays.  A launch
whose wavefront needs more than one band resets its band-wrap ring inside the
graph, so every shape can be replayed.  Runs shorter than GRAPH_MIN_ITERS
iterations, and any capture failure, use the step-by-step loop.  The same
engine serves ``softdtw_cuda.distributed.sharded_barycenter``, whose captured
iteration includes the sum of [gradient | loss] over the ranks (the library's
peer-memory exchange fused with the Adam step, or an NCCL all-reduce).
"""
from __future__ import annotations

import math

import torch

from . import _native
from .module import SoftDTW

# Use the CUDA-graph loop for CUDA tensors when it applies.
USE_CUDA_GRAPH = True
GRAPH_MIN_ITERS = 8  # shorter runs are not worth a capture
_READBACK_EVERY = 8  # replays between asynchronous loss read-backs
_GRAPH_CACHE_SIZE = 4
_graphs: dict = {}  # key -> _BaryGraph (insertion order = age)


def _cosine_lrs(lr: float, max_iter: int) -> list[float]:
    """The learning rate of every iteration and the one after the last, as
    torch's CosineAnnealingLR (T_max = max_iter, eta_min = lr / 10) sets them;
    computed by running the scheduler on a throw-away optimizer, so the values
    are the eager loop's exactly."""
    p = torch.zeros(1, requires_grad=True)
    opt = torch.optim.Adam([p], lr=lr)  # as the loop's optimizer
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=max_iter, eta_min=lr * 0.1)
    out = []
    for _ in range(max_iter):
        out.append(opt.param_groups[0]["lr"])
        opt.step()
        sched.step()
    out.append(opt.param_groups[0]["lr"])
    return out


def _early_stop_at(losses, max_iter, patience, tol):
    """Iteration at which the reference loop breaks (or None), given the loss
    of every iteration so far."""
    best = float("inf")
    stale = 0
    for it, v in enumerate(losses):
        if best - v > tol:
            best = v
            stale = 0
        else:
            stale += 1
        if stale >= patience and it > max_iter // 2:
            return it
    return None


class _BaryGraph:
    """One captured Adam iteration and the state it reads and writes.

    X (B, M, D) is read in place; the weights, the starting point (N, D), the
    Adam state, the iteration counter and the histories are persistent tensors
    that ``run`` resets before replaying.  ``reduce``, if given, is called on
    the contiguous [gradient (N*D) | loss] buffer inside the iteration (the
    sharded barycenter's all-reduce); clipping and Adam follow it.

    float32 with the fused cost (fused None or True) runs the library's
    barycenter entry points: the loss and gradient with the barycenter read
    once for all sequences and reduced over them on the device
    (``_native.barycenter_grad``), then clipping, Adam and the histories in
    one kernel (``_native.barycenter_adam``) -- a handful of launches per
    iteration.  Other configurations capture the torch loop body
    (SoftDTW module, autograd, clip_grad_norm_, capturable Adam).

    ``exchange``, if given with the library's path, is called once with the
    gradient length n and returns the peer-memory exchange of the sharded
    barycenter (``peers``, ``world``, ``rank``, ``epoch``), or None; the sum
    over ranks and the Adam step are then one kernel
    (``_native.barycenter_sync_adam``) in place of ``reduce`` and the Adam
    launch."""

    def __init__(self, X, N, gamma, fused, max_iter, lr, reduce, exchange=None):
        B, M, Dm = X.shape
        dev = X.device
        self.B, self.N, self.D, self.max_iter = B, N, Dm, max_iter
        self.X = X  # held so that its memory is not reused while the graph reads it
        self.iterations = 0
        self.lrs = _cosine_lrs(lr, max_iter)
        self.w = torch.zeros(B, dtype=X.dtype, device=dev)
        self.bary0 = torch.zeros((N, Dm), dtype=X.dtype, device=dev)
        self.lr_table = torch.tensor(self.lrs[:max_iter], dtype=torch.float32, device=dev)
        self.loss_hist = torch.zeros(max_iter, dtype=X.dtype, device=dev)
        self.bary_hist = torch.zeros((max_iter, N, Dm), dtype=X.dtype, device=dev)
        self.host_losses = torch.empty(max_iter, dtype=X.dtype, pin_memory=True)
        self.buf = torch.zeros(N * Dm + 1, dtype=X.dtype, device=dev)
        self.native = fused is not False and X.dtype == torch.float32 and X.is_contiguous()
        if self.native:
            body = self._native_body(X, gamma, reduce, exchange)
        else:
            body = self._torch_body(X, gamma, fused, reduce)

        # Warm up on a side stream (allocator, workspaces, the optimizer's
        # state, the communicator), then capture one iteration.
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                body()
        torch.cuda.current_stream(dev).wait_stream(side)
        self._reset()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            body()

    def _native_body(self, X, gamma, reduce, exchange):
        B, N, Dm, dev = self.B, self.N, self.D, X.device
        self.exchange = exchange(N * Dm) if exchange is not None else None
        ex = self.exchange
        self.bary = torch.zeros((N, Dm), dtype=torch.float32, device=dev)
        self.exp_avg = torch.zeros_like(self.bary)
        self.exp_avg_sq = torch.zeros_like(self.bary)
        self.step = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ws = _native.barycenter_workspace(B, N, X.shape[1], Dm, dev) if B > 0 else None
        bary, buf, w, ws = self.bary, self.buf, self.w, self.ws

        def body():
            if B > 0:
                _native.barycenter_grad(bary, X, w, buf, gamma, ws)
            else:
                buf.zero_()
            if ex is not None:
                _native.barycenter_sync_adam(buf, ex.peers, ex.world, ex.rank, ex.epoch, bary, self.exp_avg,
                                             self.exp_avg_sq, self.lr_table, self.step, self.loss_hist,
                                             self.bary_hist)
                return
            if reduce is not None:
                reduce(buf)
            _native.barycenter_adam(bary, self.exp_avg, self.exp_avg_sq, buf, self.lr_table, self.step,
                                    self.loss_hist, self.bary_hist)

        return body

    def _torch_body(self, X, gamma, fused, reduce):
        B, N, Dm, dev = self.B, self.N, self.D, X.device
        self.lr_t = self.lr_table[0].clone()
        self.it_t = torch.zeros(1, dtype=torch.long, device=dev)
        self.bary = torch.zeros((N, Dm), dtype=X.dtype, device=dev, requires_grad=True)
        self.bary.grad = torch.zeros_like(self.bary)
        self.opt = torch.optim.Adam([self.bary], lr=self.lr_t, capturable=True)
        loss_fn = SoftDTW(gamma=gamma, normalize=False, fused=fused)
        bary, w, buf, opt = self.bary, self.w, self.buf, self.opt

        def body():
            self.lr_t.copy_(torch.index_select(self.lr_table, 0, self.it_t)[0])
            bary.grad.zero_()
            loss = None
            if B > 0:
                d = loss_fn(bary.unsqueeze(0).expand(B, -1, -1), X)
                loss = (w * d).sum()
                loss.backward()
            if reduce is not None:
                if loss is not None:
                    buf[:-1].copy_(bary.grad.reshape(-1))
                    buf[-1:].copy_(loss.detach().reshape(1))
                else:
                    buf.zero_()
                reduce(buf)
                bary.grad.copy_(buf[:-1].view(N, Dm))
                loss_now = buf[-1:]
            else:
                loss_now = loss.detach().reshape(1)
            torch.nn.utils.clip_grad_norm_([bary], max_norm=1.0)
            opt.step()
            self.loss_hist.index_copy_(0, self.it_t, loss_now)
            self.bary_hist.index_copy_(0, self.it_t, bary.detach().unsqueeze(0))
            self.it_t.add_(1)

        return body

    def _reset(self):
        with torch.no_grad():
            self.bary.copy_(self.bary0)
            if self.native:
                self.exp_avg.zero_()
                self.exp_avg_sq.zero_()
                self.step.zero_()
                return
            self.bary.grad.zero_()
            self.it_t.zero_()
            for st in self.opt.state[self.bary].values():
                if torch.is_tensor(st):
                    st.zero_()

    def run(self, w, bary0, max_iter, early_stopping, patience, tol, verbose):
        dev = self.bary.device
        with torch.no_grad():
            self.w.copy_(w)
            self.bary0.copy_(bary0)
        self._reset()
        host_losses = self.host_losses
        done = 0
        stop = None
        while done < max_iter and stop is None:
            n = min(_READBACK_EVERY, max_iter - done)
            for _ in range(n):
                self.graph.replay()
            done += n
            if early_stopping or verbose:
                host_losses[:done].copy_(self.loss_hist[:done], non_blocking=True)
                torch.cuda.current_stream(dev).synchronize()
                if early_stopping:
                    stop = _early_stop_at(host_losses[:done].tolist(), max_iter, patience, tol)
        last = stop if stop is not None else max_iter - 1
        self.iterations = last + 1
        if verbose:
            losses = host_losses[:last + 1].tolist()
            best = float("inf")
            for it in range(last + 1):
                improvement = float("nan")
                if early_stopping:
                    improvement = best - losses[it]
                    best = losses[it] if improvement > tol else best
                if stop is not None and it == stop:
                    print(f"Early stopping at iteration {it + 1} (no improvement for {patience} iterations)")
                    break
                if (it + 1) % 20 == 0:
                    imp = f"{improvement:9.6f}" if early_stopping else "     N/A "
                    print(f"Iteration {it + 1:3d}/{max_iter} | Loss: {losses[it]:9.6f} | Improvement: {imp} | "
                          f"LR: {self.lrs[it + 1]:.2e}")
        return self.bary_hist[last].clone()


def _graph_barycenter(X, w, bary0, gamma, fused, max_iter, lr, early_stopping, patience, tol, verbose,
                      reduce=None, reduce_key=None, stats=None, exchange=None, agree=None):
    """The loop as a replayed CUDA graph (see the module docstring), captured
    once per configuration.  ``stats``, if a dict, receives the number of
    iterations run and whether this call captured the graph.  ``agree``, for
    the sharded barycenter, turns this rank's "the graph is cached" into the
    answer of all ranks (true only if true everywhere), so that every rank
    captures -- and runs the collectives of the capture's warm-up -- together."""
    N = bary0.shape[0]
    key = (X.device.index, X.data_ptr(), tuple(X.shape), X.dtype, N, float(gamma), fused, int(max_iter), float(lr),
           reduce_key)
    g = _graphs.pop(key, None)
    if agree is not None and not agree(g is not None):
        g = None
    captured = g is None
    if captured:
        g = _BaryGraph(X, N, gamma, fused, max_iter, lr, reduce, exchange)
        while len(_graphs) >= _GRAPH_CACHE_SIZE:
            _graphs.pop(next(iter(_graphs)))
    _graphs[key] = g  # newest last
    out = g.run(w, bary0, max_iter, early_stopping, patience, tol, verbose)
    if stats is not None:
        stats.update(iterations=g.iterations, captured=captured)
    return out


def clear_graph_cache() -> None:
    """Release the captured barycenter graphs (and their memory pools)."""
    _graphs.clear()


def softdtw_barycenter(
    X: torch.Tensor,
    *,
    gamma: float = 1.0,
    weights: torch.Tensor | None = None,
    max_iter: int = 100,
    lr: float = 0.1,
    init: torch.Tensor | None = None,
    device: str | torch.device | None = None,
    verbose: bool = False,
    fused: bool | None = None,
    early_stopping: bool = True,
    patience: int = 10,
    tol: float = 1e-5,
) -> torch.Tensor:
    """Barycenter (N, D) of X (B, N, D) under Soft-DTW.

    weights: (B,) non-negative, normalised to sum 1 (uniform if None).
    init:    (N, D) starting point (the weighted mean if None).
    device:  where to optimise (X's device if None).
    fused:   None = auto, True = require the fused kernels, False = never.
    early_stopping / patience / tol: stop once the loss has not improved by
             more than `tol` (absolute) for `patience` iterations, but only
             after max_iter // 2 iterations.
    """
    device = device or X.device
    X = X.to(device)
    B, N, D = X.shape
    if weights is None:
        w = torch.full((B,), 1.0 / B, device=device)
    else:
        w = weights.to(device)
        w = w / w.sum()
    if init is None:
        bary = (X * w.view(B, 1, 1)).sum(dim=0).clone()
    else:
        bary = init.clone().to(device)
    loss_fn = SoftDTW(gamma=gamma, normalize=False, fused=fused)
    if USE_CUDA_GRAPH and X.is_cuda and max_iter >= GRAPH_MIN_ITERS and B > 0:
        try:
            return _graph_barycenter(X, w, bary.detach(), gamma, fused, max_iter, lr, early_stopping, patience,
                                     tol, verbose)
        except RuntimeError:
            pass
    bary.requires_grad_(True)
    opt = torch.optim.Adam([bary], lr=lr)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=max_iter, eta_min=lr * 0.1)

    best = float("inf")
    stale = 0
    for it in range(max_iter):
        opt.zero_grad()
        d = loss_fn(bary.unsqueeze(0).expand(B, -1, -1), X)
        loss = (w * d).sum()
        loss.backward()
        torch.nn.utils.clip_grad_norm_([bary], max_norm=1.0)
        opt.step()
        sched.step()

        loss_val = loss.item()
        improvement = float("nan")
        if early_stopping:
            improvement = best - loss_val
            if improvement > tol:
                best = loss_val
                stale = 0
            else:
                stale += 1
            if stale >= patience and it > max_iter // 2:
                if verbose:
                    print(f"Early stopping at iteration {it + 1} (no improvement for {patience} iterations)")
                break

        if verbose and (it + 1) % 20 == 0:
            if torch.cuda.is_available():
                torch.cuda.synchronize()
            lr_val = opt.param_groups[0]["lr"]
            imp = f"{improvement:9.6f}" if early_stopping else "     N/A "
            print(f"Iteration {it + 1:3d}/{max_iter} | Loss: {loss_val:9.6f} | Improvement: {imp} | LR: {lr_val:.2e}")

    return bary.detach()


def softdtw_barycenter_cpu(
    X: torch.Tensor,
    *,
    gamma: float = 1.0,
    weights: torch.Tensor | None = None,
    max_iter: int = 100,
    lr: float = 0.1,
    init: torch.Tensor | None = None,
    verbose: bool = False,
    fused: bool | None = None,
    early_stopping: bool = True,
    patience: int = 10,
    tol: float = 1e-5,
) -> torch.Tensor:
    """``softdtw_barycenter`` with device="cpu"."""
    return softdtw_barycenter(X, gamma=gamma, weights=weights, max_iter=max_iter, lr=lr, init=init,
                              device="cpu", verbose=verbose, fused=fused, early_stopping=early_stopping,
                              patience=patience, tol=tol)
