"""Sharded barycenter over NCCL on two GPUs: the replayed CUDA graph (the
all-reduce of [gradient | loss] captured inside the iteration) returns, on every
rank, what the single-GPU barycenter of the concatenated shards returns, and
what the step-by-step sharded loop returns.  Runs as two spawned processes;
skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(B, N, D, seed):
    g = torch.Generator().manual_seed(seed)
    t = torch.linspace(0, 6.28, N)
    X = torch.sin(t).view(1, N, 1).repeat(B, 1, D) + 0.3 * torch.randn(B, N, D, generator=g)
    return X, torch.rand(B, generator=g) + 0.5


def _worker(rank, world, port, out_dir, early):
    from datetime import timedelta

    import torch.distributed as dist

    import softdtw_cuda.barycenters as bc
    from softdtw_cuda.distributed import shard_bounds, sharded_barycenter

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        X, w = _data(20, 48, 3, seed=11)
        lo, hi = shard_bounds(X.shape[0], rank, world)
        Xr, wr = X[lo:hi].to(dev), w[lo:hi].to(dev)
        kw = dict(gamma=1.0, max_iter=40, lr=0.1, early_stopping=early, patience=3, tol=1e-2)
        res = {}
        for graph in (True, False):
            bc.USE_CUDA_GRAPH = graph
            stats = {}
            b = sharded_barycenter(Xr, weights=wr, stats=stats, **kw)
            torch.cuda.synchronize(dev)
            res[graph] = (b.cpu(), stats["iterations"], bool(stats.get("graph")))
        bc.USE_CUDA_GRAPH = True
        # A second graph call on the same sequences replays the cached graph.
        stats = {}
        b2 = sharded_barycenter(Xr, weights=wr, stats=stats, **kw)
        torch.cuda.synchronize(dev)
        res["replay"] = (b2.cpu(), stats["iterations"], stats.get("captured"))
        torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        # Graphs holding captured NCCL calls go before the process group.
        torch.cuda.synchronize(dev)
        bc.clear_graph_cache()
        dist.destroy_process_group()


@pytest.mark.parametrize("early", [False, True])
def test_sharded_graph_two_gpus(tmp_path, early):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from softdtw_cuda import softdtw_barycenter

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), early), nprocs=2, join=True)
    X, w = _data(20, 48, 3, seed=11)
    ref = softdtw_barycenter(X.cuda(), weights=w.cuda(), gamma=1.0, max_iter=40, lr=0.1, early_stopping=early,
                             patience=3, tol=1e-2).cpu()
    outs = [torch.load(tmp_path / f"rank{r}.pt") for r in range(2)]
    for res in outs:
        b_graph, it_graph, used_graph = res[True]
        b_eager, it_eager, used_eager = res[False]
        assert used_graph and not used_eager
        assert it_graph == it_eager
        torch.testing.assert_close(b_graph, b_eager, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(b_graph, ref, rtol=1e-4, atol=1e-4)
        b_rep, it_rep, captured = res["replay"]
        assert captured is False and it_rep == it_graph
        torch.testing.assert_close(b_rep, b_graph, rtol=0, atol=0)
    torch.testing.assert_close(outs[0][True][0], outs[1][True][0], rtol=0, atol=0)
