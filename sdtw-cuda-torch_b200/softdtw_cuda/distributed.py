"""Multi-GPU Soft-DTW: batch-sharded losses and a sequence-sharded barycenter.

One process per GPU with ``torch.distributed`` (NCCL for CUDA tensors, gloo for
CPU tensors); the caller initialises the process group.  The reference package
is single-device; these functions are new and keep its single-device results:

* Loss batches.  Soft-DTW problems are independent, so each rank holds a
  contiguous slice of the batch (``shard_bounds``) and runs ``SoftDTW`` on it
  with no collective on the data path.  ``sharded_mean`` scales the local sum by
  1 / (global batch), so that the gradients of every rank's slice are exactly
  those of the global mean; the global value is one scalar all-reduce, taken
  only for reporting.
* Barycenter.  The sequence set is sharded.  Every Adam step each rank computes
  its weighted partial loss and the partial gradient of the barycenter, and one
  all-reduce (SUM) of the contiguous buffer [gradient (N*D) | loss] gives every
  rank the global gradient and loss; clipping, Adam and the cosine schedule
  then run replicated (clipping is non-linear, so it must follow the sum).  The
  weight normalisation and the initial weighted mean take one all-reduce each,
  before the loop.  The loop follows softdtw_cuda/barycenters.py:17-180 of the
  reference (Adam, cosine annealing to lr/10, clip-norm 1, early stopping after
  max_iter // 2 on the global loss).  On CUDA one iteration, all-reduce
  included, is captured in a CUDA graph and replayed (barycenters.py's graph
  engine), so a step costs no host launch overhead; every rank captures and
  replays the same collective sequence.  With the library's path the sum
  over ranks does not go through NCCL: each rank writes its [gradient | loss]
  into every rank's exchange buffer in symmetric (peer-mapped) memory over
  NVLink and sets a flag there, waits for everybody's flags, sums the slots in
  rank order and takes the Adam step -- one kernel per rank
  (``sdtw_barycenter_sync_adam_f32``); NCCL remains for the torch loop body
  and when symmetric memory is unavailable (``USE_PEER_EXCHANGE``).  The
  cached graphs hold captured NCCL calls and peer mappings: call
  ``release_graphs()`` (after a device synchronize) before
  ``torch.distributed.destroy_process_group()``, whose teardown otherwise waits
  on them.
"""
from __future__ import annotations

import time
import warnings

import torch
import torch.distributed as dist

from . import _native
from .module import SoftDTW


def _world(group=None) -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def shard_bounds(n: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous share of n items; the first n % world
    ranks take one extra item."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard(t: torch.Tensor, group=None) -> torch.Tensor:
    """This rank's slice of ``t`` along dim 0 (a view)."""
    rank, world = _world(group)
    a, b = shard_bounds(t.shape[0], rank, world)
    return t[a:b]


def _all_reduce_(t: torch.Tensor, group=None) -> torch.Tensor:
    if _world(group)[1] > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


def global_batch(local_batch: int, device, group=None) -> int:
    """Sum of the ranks' batch sizes (one integer all-reduce)."""
    t = torch.tensor([local_batch], dtype=torch.int64, device=device)
    return int(_all_reduce_(t, group).item())


def sharded_mean(losses: torch.Tensor, n_global: int) -> torch.Tensor:
    """Local contribution to the global mean: sum(losses) / n_global.  Its
    gradients are those of the global mean for this rank's slice; summing the
    returned values over ranks gives the global mean."""
    return losses.sum() / n_global


def reduce_loss(local: torch.Tensor, group=None) -> torch.Tensor:
    """Global value of per-rank contributions (sum over ranks, detached)."""
    return _all_reduce_(local.detach().clone().reshape(1), group)[0]


class ShardedSoftDTW(torch.nn.Module):
    """Batch-sharded Soft-DTW mean loss.

    ``forward(x_local, y_local)`` runs ``SoftDTW`` (same arguments as
    ``softdtw_cuda.SoftDTW``) on this rank's slice and returns
    ``sum(losses) / global_batch``.  Back-propagating it gives the global
    mean's gradients for the local slice; ``reduce_loss`` of the returned value
    is the global mean.  ``global_batch`` is taken from the ranks' slice sizes
    (one all-reduce) unless given.
    """

    def __init__(self, *, gamma: float = 1.0, bandwidth: float | None = None, normalize: bool = False,
                 dist: str = "sqeuclidean", fused: bool | None = None, group=None):
        super().__init__()
        self.loss = SoftDTW(gamma=gamma, bandwidth=bandwidth, normalize=normalize, dist=dist, fused=fused)
        self.group = group

    def forward(self, x: torch.Tensor, y: torch.Tensor, global_batch_size: int | None = None) -> torch.Tensor:
        n = global_batch_size if global_batch_size is not None else global_batch(
            x.shape[0] if x.dim() == 3 else 1, x.device, self.group)
        if x.shape[0] == 0:
            return (x.sum() + y.sum()) * 0.0
        return sharded_mean(self.loss(x, y), n)


# Sum the sharded barycenter's [gradient | loss] over ranks through peer
# memory (symmetric memory, one kernel with the Adam step) rather than NCCL.
USE_PEER_EXCHANGE = True


class _PeerExchange:
    """This rank's exchange buffer of the barycenter's sum over ranks, in
    symmetric memory mapped into every rank, and the addresses of all ranks'
    buffers (index = rank in `group`).  Creating it is collective."""

    def __init__(self, n: int, group, device):
        import torch.distributed._symmetric_memory as symm_mem

        self.rank, self.world = _world(group)
        nbytes = _native.barycenter_sync_bytes(n, self.world)
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, group if group is not None else dist.group.WORLD)
        self.peers = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=device)
        # Every buffer is zero before any rank writes into another's.
        torch.cuda.synchronize(device)
        dist.barrier(group=group)


def release_graphs() -> None:
    """Release the cached barycenter graphs (and the NCCL calls captured in
    them); to be called before destroying the process group."""
    from . import barycenters as _bc
    _bc.clear_graph_cache()


def sharded_barycenter(
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
    group=None,
    stats: dict | None = None,
) -> torch.Tensor:
    """Barycenter (N, D) of the sequences held by all ranks.

    X is this rank's shard (B_r, N, D) (B_r may be 0); weights, if given, is
    this rank's (B_r,) slice of the global weights.  Every rank returns the
    same barycenter, equal (up to the summation order) to
    ``softdtw_barycenter`` on the concatenation of the shards.  If ``stats`` is
    a dict, it receives the iteration count and the time spent in the
    all-reduce.
    """
    device = device or X.device
    X = X.to(device)
    Br, N, D = X.shape
    rank, world = _world(group)
    if weights is None:
        w = torch.ones(Br, device=device, dtype=X.dtype)
    else:
        w = weights.to(device=device, dtype=X.dtype)
    wsum = _all_reduce_(w.sum().reshape(1).clone(), group)
    w = w / wsum
    if init is None:
        bary = _all_reduce_((X * w.view(Br, 1, 1)).sum(dim=0).contiguous(), group).clone()
    else:
        bary = init.clone().to(device=device, dtype=X.dtype)
    bary.requires_grad_(True)

    from . import barycenters as _bc
    if _bc.USE_CUDA_GRAPH and X.is_cuda and max_iter >= _bc.GRAPH_MIN_ITERS:
        reduce = exchange = agree = None
        if world > 1:
            def reduce(t):
                dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)

            def agree(flag: bool) -> bool:
                t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=X.device)
                dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
                return bool(t.item())

            if USE_PEER_EXCHANGE:
                def exchange(n):
                    # Symmetric memory unavailable (it fails on every rank
                    # before any peer access): the NCCL all-reduce instead.
                    try:
                        return _PeerExchange(n, group, X.device)
                    except (RuntimeError, ImportError, AttributeError) as err:
                        warnings.warn(f"softdtw_cuda: peer-memory exchange unavailable ({err}); using NCCL")
                        return None
        t0 = time.time()
        info = {}
        res = _bc._graph_barycenter(X, w, bary.detach(), gamma, fused, max_iter, lr, early_stopping, patience, tol,
                                    verbose and rank == 0, reduce=reduce,
                                    reduce_key=("sum", id(group), world, exchange is not None),
                                    stats=info, exchange=exchange, agree=agree)
        if stats is not None:
            # The all-reduce runs inside the graph, where it cannot be timed
            # apart from the iteration: allreduce_s is None.
            stats.update(iterations=info["iterations"], allreduce_s=None, wall_s=time.time() - t0, world=world,
                         graph=True, captured=info["captured"])
        return res

    loss_fn = SoftDTW(gamma=gamma, normalize=False, fused=fused)
    opt = torch.optim.Adam([bary], lr=lr)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=max_iter, eta_min=lr * 0.1)
    # [gradient | loss] reduced in one collective per step.
    buf = torch.empty(N * D + 1, device=device, dtype=X.dtype)
    reduce_s = 0.0
    on_gpu = buf.is_cuda
    ev = []  # (start, end) CUDA events around each all-reduce, read once at the end

    t0 = time.time()
    best = float("inf")
    stale = 0
    it = -1
    for it in range(max_iter):
        opt.zero_grad()
        if Br > 0:
            d = loss_fn(bary.unsqueeze(0).expand(Br, -1, -1), X)
            loss = (w * d).sum()
            loss.backward()
            buf[:-1].copy_(bary.grad.reshape(-1))
            buf[-1:].copy_(loss.detach().reshape(1))
        else:
            buf.zero_()
        if world > 1:
            if on_gpu:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
                e1.record()
                ev.append((e0, e1))
            else:
                r0 = time.perf_counter()
                dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
                reduce_s += time.perf_counter() - r0
        if bary.grad is None:
            bary.grad = torch.empty_like(bary)
        bary.grad.copy_(buf[:-1].view(N, D))
        torch.nn.utils.clip_grad_norm_([bary], max_norm=1.0)
        opt.step()
        sched.step()

        need_value = early_stopping or (verbose and (it + 1) % 20 == 0)
        if not need_value:
            continue
        loss_val = float(buf[-1].item())
        improvement = float("nan")
        if early_stopping:
            improvement = best - loss_val
            if improvement > tol:
                best = loss_val
                stale = 0
            else:
                stale += 1
            if stale >= patience and it > max_iter // 2:
                if verbose and rank == 0:
                    print(f"Early stopping at iteration {it + 1} (no improvement for {patience} iterations)")
                break
        if verbose and rank == 0 and (it + 1) % 20 == 0:
            lr_val = opt.param_groups[0]["lr"]
            imp = f"{improvement:9.6f}" if early_stopping else "     N/A "
            print(f"Iteration {it + 1:3d}/{max_iter} | Loss: {loss_val:9.6f} | Improvement: {imp} | LR: {lr_val:.2e}")

    if stats is not None:
        if ev:
            torch.cuda.synchronize(buf.device)
            reduce_s = sum(a.elapsed_time(b) for a, b in ev) / 1e3
        stats.update(iterations=it + 1, allreduce_s=reduce_s, wall_s=time.time() - t0, world=world)
    return bary.detach()
