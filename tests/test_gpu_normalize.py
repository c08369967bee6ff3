"""normalize=True reads x and y in place (sdtw_*_norm_f32): the three pairs
(x, y), (x, x), (y, y) of every problem without concatenated copies.

Checked against the concatenation of softdtw_cuda/module.py:99-111 of the
reference (the same 3B problems through the plain x/y entry points), on every
kernel route of the library, and against the oracle on a small case.  The
losses are bit-identical (the same kernels on the same problems); the
gradients differ only in the order the three contributions are added:
rtol 1e-5, atol 1e-6.
"""
import numpy as np
import pytest
import torch

from _tol import assert_grad_close, assert_loss_close, noise_floor
from oracle import oracle as O
from softdtw_cuda import SoftDTW, _native
from softdtw_cuda.autograd import SoftDTWSqEuclidAutograd
from softdtw_cuda.autograd_xy import SoftDTWXYAutograd

pytestmark = pytest.mark.gpu

# (B, N, dim, bandwidth, rows per lane override): the route it exercises.
CASES = [
    (3, 40, 3, None, 0),     # costs inside the forward (dense rows), gradients on the FP32 pipes
    (2, 70, 16, None, 0),    # 16 features: the widest in-forward cost and FP32 gradient
    (2, 100, 64, None, 0),   # one 128-row tile: cost table, row-major tensor-core gradient
    (2, 300, 64, None, 0),   # wavefront-layout tensor-core gradient, chunked transposes
    (2, 150, 5, None, 0),    # 5 features: scalar cost loads, no tensor-core cost
    (2, 120, 8, 9.0, 0),     # Sakoe-Chiba band
    (2, 200, 24, None, 2),   # two rows per lane: score store, clamp mask in the gradient
]


def _pair(x, y, *, fused, gamma, bw, w, in_place, need_y=True):
    xt = x.clone().requires_grad_(True)
    yt = y.clone().requires_grad_(need_y)
    B = x.shape[0]
    if in_place:
        out = SoftDTW(gamma=gamma, bandwidth=bw, normalize=True, fused=fused)(xt, yt)
    else:
        xs = torch.cat([xt, xt, yt], dim=0)
        ys = torch.cat([yt, xt, yt], dim=0)
        fn = SoftDTWXYAutograd if fused else SoftDTWSqEuclidAutograd
        o_xy, o_xx, o_yy = fn.apply(xs, ys, gamma, bw).split(B, dim=0)
        out = o_xy - 0.5 * (o_xx + o_yy)
    (out * w).sum().backward()
    torch.cuda.synchronize()
    _native.check_status()
    return out.detach(), xt.grad, (yt.grad if need_y else None)


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("B,N,dim,bw,k", CASES)
def test_in_place_matches_concatenation(B, N, dim, bw, k, fused):
    g = torch.Generator().manual_seed(N * 31 + dim)
    x = torch.randn(B, N, dim, generator=g).cuda()
    y = torch.randn(B, N, dim, generator=g).cuda()
    w = torch.rand(B, generator=g).cuda() + 0.5
    _native.set_plan_override(0, 0, k)
    try:
        a = _pair(x, y, fused=fused, gamma=0.7, bw=bw, w=w, in_place=True)
        b = _pair(x, y, fused=fused, gamma=0.7, bw=bw, w=w, in_place=False)
    finally:
        _native.set_plan_override(0, 0, 0)
    assert torch.equal(a[0], b[0]), "losses differ from the concatenated batch"
    for ours, ref, what in ((a[1], b[1], "grad_x"), (a[2], b[2], "grad_y")):
        assert torch.isfinite(ours).all()
        torch.testing.assert_close(ours, ref, rtol=1e-5, atol=1e-6, msg=lambda m: f"{what}: {m}")


@pytest.mark.parametrize("fused", [False, True])
def test_in_place_x_only(fused):
    """y without gradient: x still gets both sides of its self pair."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 90, 12, generator=g).cuda()
    y = torch.randn(3, 90, 12, generator=g).cuda()
    w = torch.ones(3, device="cuda")
    a = _pair(x, y, fused=fused, gamma=1.0, bw=None, w=w, in_place=True, need_y=False)
    b = _pair(x, y, fused=fused, gamma=1.0, bw=None, w=w, in_place=False, need_y=False)
    assert torch.equal(a[0], b[0])
    torch.testing.assert_close(a[1], b[1], rtol=1e-5, atol=1e-6)


def test_in_place_vs_oracle():
    rng = np.random.default_rng(21)
    x = rng.standard_normal((3, 50, 6)).astype(np.float32)
    y = rng.standard_normal((3, 50, 6)).astype(np.float32)
    gout = np.array([1.0, -0.5, 2.0])
    for fused in (False, True):
        xt = torch.tensor(x, device="cuda", requires_grad=True)
        yt = torch.tensor(y, device="cuda", requires_grad=True)
        out = SoftDTW(gamma=0.5, normalize=True, fused=fused)(xt, yt)
        (out * torch.tensor(gout, device="cuda", dtype=torch.float32)).sum().backward()
        torch.cuda.synchronize()
        kw = dict(gamma=0.5, normalize=True, fused=fused, grad_out=gout)
        o32, gx32, gy32 = O.loss_and_grads(x, y, **kw)
        o64, gx64, gy64 = O.loss_and_grads(x, y, precision="float64", **kw)
        assert_loss_close(out.detach().cpu().numpy(), o64, rtol=1e-4, what="normalized loss vs float64")
        fx, fy = noise_floor(gx32, gx64), noise_floor(gy32, gy64)
        assert_grad_close(xt.grad.cpu().numpy(), gx64, floor=fx, what="grad_x vs float64")
        assert_grad_close(yt.grad.cpu().numpy(), gy64, floor=fy, what="grad_y vs float64")


@pytest.mark.parametrize("fused", [False, True])
def test_in_place_needs_no_concatenated_copies(fused):
    """The forward's peak memory stays below the concatenation's by most of
    the 2 x 3B x N x dim floats it copies."""
    B, N, dim = 8, 512, 128
    g = torch.Generator().manual_seed(1)
    x = torch.randn(B, N, dim, generator=g).cuda()
    y = torch.randn(B, N, dim, generator=g).cuda()
    copies = 2 * 3 * B * N * dim * 4
    peaks = []
    for in_place in (True, False):
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        xt = x.clone().requires_grad_(True)
        yt = y.clone().requires_grad_(True)
        if in_place:
            out = SoftDTW(gamma=1.0, normalize=True, fused=fused)(xt, yt)
        else:
            xs, ys = torch.cat([xt, xt, yt]), torch.cat([yt, xt, yt])
            fn = SoftDTWXYAutograd if fused else SoftDTWSqEuclidAutograd
            out = fn.apply(xs, ys, 1.0, None)
        torch.cuda.synchronize()
        peaks.append(torch.cuda.max_memory_allocated() - base)
        del out, xt, yt
    assert peaks[0] <= peaks[1] - 0.9 * copies, f"peaks {peaks}, copies {copies}"


def test_in_place_half_inputs():
    """bfloat16 x, y: the losses equal the concatenated batch's; the gradients,
    computed in float32 and rounded once, are within bfloat16 rounding of the
    float32 run on the same (rounded) inputs."""
    g = torch.Generator().manual_seed(9)
    x = torch.randn(2, 80, 24, generator=g).to(torch.bfloat16).cuda()
    y = torch.randn(2, 80, 24, generator=g).to(torch.bfloat16).cuda()
    w = torch.ones(2, device="cuda")
    for fused in (False, True):
        a = _pair(x, y, fused=fused, gamma=1.0, bw=None, w=w, in_place=True)
        b = _pair(x, y, fused=fused, gamma=1.0, bw=None, w=w, in_place=False)
        ref = _pair(x.float(), y.float(), fused=fused, gamma=1.0, bw=None, w=w, in_place=True)
        assert a[0].dtype == torch.bfloat16 and torch.equal(a[0], b[0])
        for ours, r in ((a[1], ref[1]), (a[2], ref[2])):
            assert ours.dtype == torch.bfloat16
            torch.testing.assert_close(ours.float(), r, rtol=8e-3, atol=8e-3 * float(r.abs().max()))


def test_norm_entry_points_reject_missing_gradient():
    """The normalized backward writes both gradients: a null one is refused
    before any launch."""
    B, N, dim = 2, 40, 4
    x = torch.randn(B, N, dim, device="cuda")
    y = torch.randn(B, N, dim, device="cuda")
    out, score = _native.forward_xy_norm(x, y, 1.0, -1.0)
    L = _native.lib()
    ws = torch.empty(L.sdtw_workspace_bytes_norm(B, N, dim), dtype=torch.uint8, device="cuda")
    gx = torch.empty_like(x)
    stream = _native._stream(x.device)
    rc = L.sdtw_backward_xy_norm_f32(_native._ptr(x), _native._ptr(y), _native._ptr(score), None, _native._ptr(gx),
                                     None, B, N, dim, 1.0, -1.0, _native._ptr(ws), ws.numel(), stream)
    assert rc == 1 and b"both gradients" in L.sdtw_last_error_message()
    rc = L.sdtw_backward_xy_norm_f32(_native._ptr(x), _native._ptr(y), _native._ptr(score), None, _native._ptr(gx),
                                     _native._ptr(gx), B, N, dim, 1.0, -1.0, _native._ptr(ws), 16, stream)
    assert rc == 1 and b"workspace" in L.sdtw_last_error_message()
    torch.cuda.synchronize()
    _native.check_status()
