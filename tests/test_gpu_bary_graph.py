"""The CUDA-graph barycenter loop returns what the step-by-step loop returns
(same stopping iteration, same progress messages, barycenter to float32
rounding of the capturable Adam arithmetic)."""
import contextlib
import io

import pytest
import torch

import softdtw_cuda.barycenters as bc
from softdtw_cuda import softdtw_barycenter

pytestmark = pytest.mark.gpu


def _data(B, N, D, seed):
    g = torch.Generator().manual_seed(seed)
    t = torch.linspace(0, 6.28, N)
    X = torch.sin(t).view(1, N, 1).repeat(B, 1, D) + 0.3 * torch.randn(B, N, D, generator=g)
    return X.cuda(), (torch.rand(B, generator=g) + 0.5).cuda()


def _run(graph, X, **kw):
    old = bc.USE_CUDA_GRAPH
    bc.USE_CUDA_GRAPH = graph
    buf = io.StringIO()
    try:
        with contextlib.redirect_stdout(buf):
            b = softdtw_barycenter(X, **kw)
    finally:
        bc.USE_CUDA_GRAPH = old
    torch.cuda.synchronize()
    return b, buf.getvalue()


@pytest.mark.parametrize("early,weighted,fused", [(False, False, None), (True, True, None), (True, False, False)])
def test_graph_loop_matches_step_loop(early, weighted, fused):
    X, w = _data(16, 40, 3, seed=3)
    kw = dict(gamma=1.0, max_iter=60, lr=0.1, early_stopping=early, patience=3, tol=1e-2, verbose=True,
              weights=w if weighted else None, fused=fused)
    assert kw["max_iter"] >= bc.GRAPH_MIN_ITERS
    b_graph, out_graph = _run(True, X, **kw)
    b_eager, out_eager = _run(False, X, **kw)
    torch.testing.assert_close(b_graph, b_eager, rtol=1e-4, atol=1e-5)
    # Same messages; the printed losses agree to the digits shown except for
    # float rounding of the last digit, so compare the message skeletons.
    strip = lambda s: [ln.split("| Loss")[0] if ln.startswith("Iteration") else ln for ln in s.splitlines()]
    assert strip(out_graph) == strip(out_eager)


def test_graph_cache_reuse_and_multiband():
    """A second call with the same configuration replays the cached graph with
    the new weights and starting point; a shape whose wavefront runs in many
    bands (forced plan) replays correctly (its band-wrap ring is reset inside
    the graph)."""
    from softdtw_cuda import _native
    bc.clear_graph_cache()
    X, w = _data(12, 70, 3, seed=5)
    kw = dict(gamma=1.0, max_iter=24, lr=0.1, early_stopping=False)
    b1, _ = _run(True, X, weights=w, **kw)
    n_cached = len(bc._graphs)
    b2, _ = _run(True, X, weights=w.flip(0), init=X[0], **kw)
    assert len(bc._graphs) == n_cached  # replayed, not captured again
    torch.testing.assert_close(b1, _run(False, X, weights=w, **kw)[0], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(b2, _run(False, X, weights=w.flip(0), init=X[0], **kw)[0], rtol=1e-4, atol=1e-5)
    _native.set_plan_override(1, 1, 1)  # one stripe per CTA, one CTA per cluster: 3 bands at N = 70
    try:
        assert _native.plan_info(12, 70, 70)["bands"] > 1
        bc.clear_graph_cache()
        b3, _ = _run(True, X, weights=w, **kw)
        b4, _ = _run(True, X, weights=w, **kw)
        b5, _ = _run(False, X, weights=w, **kw)
    finally:
        _native.set_plan_override(0, 0, 0)
        bc.clear_graph_cache()
    torch.testing.assert_close(b3, b5, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(b4, b5, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("B,N,M,D", [(16, 40, 40, 3), (7, 33, 50, 8), (5, 70, 20, 5), (6, 24, 30, 20), (3, 1, 9, 2)])
def test_native_barycenter_grad_matches_autograd(B, N, M, D):
    """sdtw_barycenter_grad_f32 (barycenter read once for every sequence, the
    gradient and the loss reduced on the device) equals the torch formulation
    of barycenters.py:122-131: expand, SoftDTW, weighted sum, backward."""
    from softdtw_cuda import SoftDTW, _native
    g = torch.Generator().manual_seed(B * 1000 + N)
    X = torch.randn(B, M, D, generator=g).cuda()
    bary = torch.randn(N, D, generator=g).cuda()
    w = (torch.rand(B, generator=g) + 0.5).cuda()
    w = w / w.sum()
    buf = torch.empty(N * D + 1, device="cuda")
    ws = _native.barycenter_workspace(B, N, M, D, X.device)
    _native.barycenter_grad(bary, X, w, buf, 0.7, ws)
    b = bary.clone().requires_grad_(True)
    loss = (w * SoftDTW(gamma=0.7, fused=True)(b.unsqueeze(0).expand(B, -1, -1), X)).sum()
    loss.backward()
    torch.testing.assert_close(buf[-1], loss.detach(), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(buf[:-1].view(N, D), b.grad, rtol=1e-4, atol=1e-5)
    # Bit-reproducible.
    buf2 = torch.empty_like(buf)
    _native.barycenter_grad(bary, X, w, buf2, 0.7, ws)
    assert torch.equal(buf, buf2)


def test_native_barycenter_adam_matches_torch():
    """sdtw_barycenter_adam_f32 = clip_grad_norm_(max_norm=1) + torch Adam with
    the cosine-annealed learning rate, over several steps."""
    from softdtw_cuda import _native
    g = torch.Generator().manual_seed(9)
    n, steps = 37, 12
    lrs = bc._cosine_lrs(0.1, steps)
    p = torch.randn(n, generator=g).cuda()
    ref = p.clone().requires_grad_(True)
    opt = torch.optim.Adam([ref], lr=0.1)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=steps, eta_min=0.01)
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    step = torch.zeros(1, dtype=torch.int32, device="cuda")
    lr_table = torch.tensor(lrs[:steps], device="cuda")
    loss_hist = torch.zeros(steps, device="cuda")
    hist = torch.zeros(steps, n, device="cuda")
    for it in range(steps):
        grad = torch.randn(n, generator=g).cuda() * (3.0 if it % 2 else 0.2)  # clipped and unclipped steps
        buf = torch.cat([grad, torch.tensor([float(it)], device="cuda")])
        _native.barycenter_adam(p, m, v, buf, lr_table, step, loss_hist, hist)
        ref.grad = grad.clone()
        torch.nn.utils.clip_grad_norm_([ref], max_norm=1.0)
        opt.step()
        sched.step()
        torch.testing.assert_close(p, ref.detach(), rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(hist[it], ref.detach(), rtol=1e-5, atol=1e-6)
    assert int(step.item()) == steps
    assert loss_hist.tolist() == [float(i) for i in range(steps)]
    # Past max_iter the step does nothing.
    before = p.clone()
    _native.barycenter_adam(p, m, v, buf, lr_table, step, loss_hist, hist)
    assert torch.equal(p, before) and int(step.item()) == steps
