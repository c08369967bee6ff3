"""Multi-process host logic of softdtw_cuda.distributed on CPU (gloo, world size 2).

Each test spawns two ranks that hold slices of one batch; their results must
equal the single-process package run on the whole batch: the batch-sharded
mean loss and its per-sample gradients, and the sequence-sharded barycenter
(one all-reduce of [gradient | loss] per Adam step).
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from softdtw_cuda import SoftDTW, softdtw_barycenter
from softdtw_cuda.distributed import ShardedSoftDTW, reduce_loss, shard, shard_bounds, sharded_barycenter

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, port):
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=timedelta(seconds=60))
    torch.set_num_threads(1)
    return dist


def _loss_worker(rank, port, x, y, out_dir):
    dist = _init(rank, port)
    try:
        xs = shard(x).clone().requires_grad_(True)
        ys = shard(y).clone().requires_grad_(True)
        local = ShardedSoftDTW(gamma=0.5, fused=False)(xs, ys)
        local.backward()
        glob = reduce_loss(local)
        np.savez(os.path.join(out_dir, f"loss{rank}.npz"), loss=glob.numpy(), gx=xs.grad.numpy(),
                 gy=ys.grad.numpy())
    finally:
        dist.destroy_process_group()


def _bary_worker(rank, port, X, w, kw, out_dir):
    dist = _init(rank, port)
    try:
        stats = {}
        ws = shard(w) if w is not None else None
        b = sharded_barycenter(shard(X), weights=ws, stats=stats, **kw)
        np.savez(os.path.join(out_dir, f"bary{rank}.npz"), b=b.numpy(), it=stats["iterations"])
    finally:
        dist.destroy_process_group()


def _spawn(fn, *args):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=fn, args=(r, port) + args) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_shard_bounds_cover_every_item_once():
    for n in range(0, 13):
        for world in range(1, 6):
            spans = [shard_bounds(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


@pytest.mark.parametrize("B", [6, 5])
def test_batch_sharded_loss_matches_single_process(B):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(B, 20, 3, generator=g)
    y = torch.randn(B, 17, 3, generator=g)
    with tempfile.TemporaryDirectory() as d:
        _spawn(_loss_worker, x, y, d)
        parts = [dict(np.load(os.path.join(d, f"loss{r}.npz"))) for r in range(WORLD)]
    xr = x.clone().requires_grad_(True)
    yr = y.clone().requires_grad_(True)
    ref = SoftDTW(gamma=0.5, fused=False)(xr, yr).mean()
    ref.backward()
    for p in parts:  # every rank sees the same global mean
        np.testing.assert_allclose(p["loss"], ref.item(), rtol=1e-6)
    np.testing.assert_allclose(np.concatenate([p["gx"] for p in parts]), xr.grad.numpy(), rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(np.concatenate([p["gy"] for p in parts]), yr.grad.numpy(), rtol=1e-6, atol=1e-9)


@pytest.mark.parametrize("B,weighted,early", [(6, False, False), (5, True, True), (1, False, False)])
def test_sharded_barycenter_matches_single_process(B, weighted, early):
    """B=1 leaves rank 1 with an empty shard."""
    g = torch.Generator().manual_seed(7)
    t = torch.linspace(0, 6.28, 24)
    X = torch.sin(t).view(1, 24, 1).repeat(B, 1, 2) + 0.3 * torch.randn(B, 24, 2, generator=g)
    w = torch.rand(B, generator=g) + 0.5 if weighted else None
    kw = dict(gamma=1.0, max_iter=30, lr=0.1, early_stopping=early, patience=3, tol=1e-2)
    with tempfile.TemporaryDirectory() as d:
        _spawn(_bary_worker, X, w, kw, d)
        parts = [dict(np.load(os.path.join(d, f"bary{r}.npz"))) for r in range(WORLD)]
    ref = softdtw_barycenter(X, weights=w, **kw).numpy()
    assert np.array_equal(parts[0]["b"], parts[1]["b"])  # replicated update: identical on every rank
    assert int(parts[0]["it"]) == int(parts[1]["it"])
    np.testing.assert_allclose(parts[0]["b"], ref, rtol=1e-4, atol=1e-5)
