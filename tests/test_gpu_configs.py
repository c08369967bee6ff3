"""GPU parity at the benchmark configurations and on the public entry points
the other parity files do not reach.

* C3, C4a and C4b at their full shapes and value distributions (the seeded
  synthetic data bench.py times), with the oracle run on a few of the problems;
* ``distances.sqeuclidean`` / ``pairwise_distance`` on CUDA (float32, float16,
  bfloat16) and their gradients, against the reference's torch expression;
* the reference-named launcher wrappers of the fused path;
* the CUDA barycenter (CUDA-graph loop and step-by-step loop) against the
  reference's own barycenter output (tests/golden/bary.npz);
* float16 / bfloat16 inputs against the oracle run on the same rounded inputs.

Tolerances as everywhere (see conftest.py): loss 1e-5 relative; gradients
rtol 1e-4 / atol 1e-6 plus the reference's own float32 noise floor.
"""
import contextlib
import io

import numpy as np
import pytest
import torch

import bench
import softdtw_cuda.barycenters as bc
from _tol import assert_grad_close, assert_loss_close, noise_floor
from conftest import golden, golden_manifest
from oracle import oracle as O
from softdtw_cuda import SoftDTW, _native, softdtw_barycenter
from softdtw_cuda.cuda import launcher
from softdtw_cuda.distances import _sqeuclidean_torch, pairwise_distance, sqeuclidean

pytestmark = pytest.mark.gpu


def _gpu_run(x, y, *, gamma, normalize=False, fused=None):
    """Mean-reduced loss (the benchmark step): per-problem outputs and grads."""
    xt = torch.tensor(x, device="cuda", requires_grad=True)
    yt = torch.tensor(y, device="cuda", requires_grad=True)
    out = SoftDTW(gamma=gamma, normalize=normalize, fused=fused)(xt, yt)
    out.mean().backward()
    torch.cuda.synchronize()
    _native.check_status()
    return out.detach().cpu().numpy(), xt.grad.cpu().numpy(), yt.grad.cpu().numpy()


def _check_subset(x, y, out, gx, gy, idx, *, gamma, normalize=False, fused=False):
    """Problems `idx` of a batch of B against the oracle (their losses and
    gradients do not depend on the other problems; the mean's 1/B is grad_out)."""
    B = x.shape[0]
    xs, ys = x[idx], y[idx]
    g = np.full(len(idx), 1.0 / B)
    kw = dict(gamma=gamma, normalize=normalize, fused=fused, grad_out=g)
    o32, gx32, gy32 = O.loss_and_grads(xs, ys, **kw)
    o64, gx64, gy64 = O.loss_and_grads(xs, ys, precision="float64", **kw)
    assert_loss_close(out[idx], o32, what="loss vs reference")
    assert_loss_close(out[idx], o64, what="loss vs float64")
    fx, fy = noise_floor(gx32, gx64), noise_floor(gy32, gy64)
    assert_grad_close(gx[idx], gx64, floor=fx, what="grad_x vs float64")
    assert_grad_close(gy[idx], gy64, floor=fy, what="grad_y vs float64")
    assert_grad_close(gx[idx], gx32, floor=2 * fx, what="grad_x vs reference")
    assert_grad_close(gy[idx], gy32, floor=2 * fy, what="grad_y vs reference")


def test_c3_long_sequences_fused():
    """C3: B=16, N=M=4096, D=8, gamma=0.1, sines and a time-warped copy; the
    default (fused) CUDA path over all 16 problems, the oracle on 2."""
    B, N, M, Dm, gamma, *_ = bench.WORKLOADS["c3"]
    x, y = bench.make_data("c3", B, N, M, Dm, seed=1234)
    out, gx, gy = _gpu_run(x, y, gamma=gamma)
    assert np.isfinite(out).all() and np.isfinite(gx).all() and np.isfinite(gy).all()
    _check_subset(x, y, out, gx, gy, [0, 9], gamma=gamma, fused=True)


@pytest.mark.parametrize("fused", [False, True])
def test_c4a_unequal_lengths(fused):
    """C4a: B=64, N=1024, M=768, D=128, gamma=1 (unfused is the config's mode);
    the oracle on 4 of the 64 problems."""
    B, N, M, Dm, gamma, *_ = bench.WORKLOADS["c4a"]
    x, y = bench.make_data("c4a", B, N, M, Dm, seed=1234)
    out, gx, gy = _gpu_run(x, y, gamma=gamma, fused=fused)
    _check_subset(x, y, out, gx, gy, [0, 17, 42, 63], gamma=gamma, fused=fused)


@pytest.mark.parametrize("fused", [False, True])
def test_c4b_normalize(fused):
    """C4b: normalize=True on B=64, N=M=1024, D=128 (192 problems in one launch
    of each kernel); the oracle on 2 of the 64 (xy, xx, yy) triples."""
    B, N, M, Dm, gamma, *_ = bench.WORKLOADS["c4b"]
    x, y = bench.make_data("c4b", B, N, M, Dm, seed=1234)
    out, gx, gy = _gpu_run(x, y, gamma=gamma, normalize=True, fused=fused)
    _check_subset(x, y, out, gx, gy, [3, 50], gamma=gamma, normalize=True, fused=fused)


# ------------------------------------------------------------------ distances
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=str)
@pytest.mark.parametrize("dim", [1, 8, 16, 33, 64, 65, 128])
def test_sqeuclidean_cuda_matches_reference_expression(dim, dtype):
    """distances.sqeuclidean on CUDA against the reference's expression
    (distances.py:6-28) evaluated in float64 on the same (rounded) inputs, N != M;
    gradients of sum(W * D) against torch autograd of that expression.  Feature
    counts of 16 and more that are multiples of 4 take the tensor-core cost."""
    g = torch.Generator().manual_seed(dim)
    x = torch.randn(3, 37, dim, generator=g).to(dtype)
    y = torch.randn(3, 29, dim, generator=g).to(dtype)
    W = torch.rand(3, 37, 29, generator=g)
    xd = x.cuda().requires_grad_(True)
    yd = y.cuda().requires_grad_(True)
    D = sqeuclidean(xd, yd)
    assert D.dtype == dtype and D.shape == (3, 37, 29)
    (D.float() * W.cuda()).sum().backward()
    x64 = x.double().requires_grad_(True)
    y64 = y.double().requires_grad_(True)
    D64 = _sqeuclidean_torch(x64, y64)
    (D64 * W.double()).sum().backward()
    # The library computes in float32 and rounds the result to the input dtype.
    scale = float(D64.detach().abs().max())
    out_tol = {torch.float32: 2e-6, torch.float16: 1e-3, torch.bfloat16: 8e-3}[dtype]
    np.testing.assert_allclose(D.detach().float().cpu().numpy(), D64.detach().numpy(), rtol=out_tol,
                               atol=out_tol * scale + 1e-6 * dim)
    gscale = max(float(x64.grad.abs().max()), float(y64.grad.abs().max()))
    np.testing.assert_allclose(xd.grad.float().cpu().numpy(), x64.grad.numpy(), rtol=out_tol,
                               atol=out_tol * gscale + 1e-5)
    np.testing.assert_allclose(yd.grad.float().cpu().numpy(), y64.grad.numpy(), rtol=out_tol,
                               atol=out_tol * gscale + 1e-5)


@pytest.mark.parametrize("N,M,dim", [(300, 200, 64), (129, 257, 16), (128, 128, 128)])
def test_sqeuclidean_tensor_core_tiles(N, M, dim):
    """The tensor-core cost across several 128 x 128 tiles and ragged edges,
    against the reference's expression in float64."""
    g = torch.Generator().manual_seed(N + M + dim)
    x = torch.randn(2, N, dim, generator=g)
    y = torch.randn(2, M, dim, generator=g)
    D = sqeuclidean(x.cuda(), y.cuda())
    D64 = _sqeuclidean_torch(x.double(), y.double())
    scale = float(D64.abs().max())
    np.testing.assert_allclose(D.cpu().numpy(), D64.numpy(), rtol=2e-6, atol=2e-6 * scale)


def test_sqeuclidean_clamp_mask_and_pairwise_name():
    """Identical rows give a clamped (zero) cost and no gradient through it;
    pairwise_distance resolves the reference's dist names to the same kernel."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 20, 5, generator=g)
    y = x[:, :15].clone() + 0.0
    y[:, 5:] += torch.randn(2, 10, 5, generator=g)
    xd = x.cuda().requires_grad_(True)
    D = pairwise_distance(xd, y.cuda(), dist="SqEuclidean")
    assert (D >= 0).all()
    ref = _sqeuclidean_torch(x.double(), y.double())
    np.testing.assert_allclose(D.detach().cpu().numpy(), ref.numpy(), rtol=2e-6, atol=2e-5)
    D.sum().backward()
    xr = x.double().requires_grad_(True)
    _sqeuclidean_torch(xr, y.double()).sum().backward()
    np.testing.assert_allclose(xd.grad.cpu().numpy(), xr.grad.numpy(), rtol=1e-4, atol=1e-4)


# ------------------------------------------------------------------ launcher wrappers
@pytest.mark.parametrize("bandwidth", [-1.0, 6.0])
def test_fused_launcher_wrappers_vs_oracle(bandwidth):
    """softdtw_forward_cuda_fused_sqeuclid / softdtw_backward_cuda_fused_sqeuclid
    (launcher.py:33-162): R in the reference layout and E, against the oracle's
    tables for the direct-form (fused) cost."""
    rng = np.random.default_rng(8)
    X = rng.standard_normal((3, 40, 4)).astype(np.float32)
    Y = rng.standard_normal((3, 33, 4)).astype(np.float32)
    out, R = launcher.softdtw_forward_cuda_fused_sqeuclid(torch.tensor(X, device="cuda"),
                                                          torch.tensor(Y, device="cuda"), 0.7, bandwidth)
    E = launcher.softdtw_backward_cuda_fused_sqeuclid(torch.tensor(X, device="cuda"), torch.tensor(Y, device="cuda"),
                                                       R, 0.7, bandwidth)
    torch.cuda.synchronize()
    _native.check_status()
    bw = None if bandwidth <= 0 else bandwidth
    D = O.cost_direct(X, Y)
    o_ref, R_ref, _ = O.forward(D.astype(np.float32), 0.7, bw)
    assert R.shape == (3, 42, 35) and R.dtype == torch.float32
    assert_loss_close(out.cpu().numpy(), o_ref, what="fused launcher loss")
    Rn = R.cpu().numpy()
    fin = np.isfinite(R_ref)
    assert np.array_equal(np.isfinite(Rn), fin)
    np.testing.assert_allclose(Rn[fin], R_ref[fin], rtol=2e-6, atol=2e-6 * np.abs(R_ref[fin]).max())
    _, R64, _ = O.forward(D, 0.7, bw)
    E64 = O.backward(D, R64, 0.7, bw)
    E32 = O.backward(D.astype(np.float32), R_ref, 0.7, bw)
    floor = noise_floor(E32, E64)
    assert_grad_close(E.cpu().numpy(), E64, floor=floor + 1e-5, what="E vs float64")


# ------------------------------------------------------------------ barycenter
def _bary(graph, X, **kw):
    old = bc.USE_CUDA_GRAPH
    bc.USE_CUDA_GRAPH = graph
    try:
        with contextlib.redirect_stdout(io.StringIO()):
            b = softdtw_barycenter(X, **kw)
    finally:
        bc.USE_CUDA_GRAPH = old
    torch.cuda.synchronize()
    _native.check_status()
    return b.cpu().numpy()


@pytest.mark.parametrize("graph", [True, False], ids=["graph", "steps"])
@pytest.mark.parametrize("fused", [False, None], ids=["unfused", "fused"])
def test_cuda_barycenter_matches_reference_output(graph, fused):
    """softdtw_barycenter on CUDA (replayed CUDA graph, and step by step) against
    the reference's barycenter of the same sequences (barycenters.py:17-180 run
    in the reference itself; 10 Adam iterations, lr 0.1, gamma 1), unweighted
    and weighted.  The reference's sequence used the expanded cost; the fused
    path's direct-form cost agrees with it to float32 rounding."""
    m = golden_manifest()["bary"]
    z = golden("bary")
    X = torch.tensor(z["X"], device="cuda")
    kw = dict(gamma=m["gamma"], max_iter=m["max_iter"], lr=m["lr"], early_stopping=m["early_stopping"], fused=fused)
    b = _bary(graph, X, **kw)
    np.testing.assert_allclose(b, z["bary"], rtol=1e-4, atol=1e-5)
    bw = _bary(graph, X, weights=torch.tensor(z["weights"], device="cuda"), **kw)
    np.testing.assert_allclose(bw, z["bary_w"], rtol=1e-4, atol=1e-5)


# ------------------------------------------------------------------ half inputs
@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=str)
def test_half_inputs_vs_oracle(dtype, fused):
    """float16 / bfloat16 x, y: the library computes in float32 and returns the
    input dtype, so the reference is the oracle run on the same rounded inputs,
    compared after rounding to that dtype (half an ulp of the output dtype
    added to the loss and gradient tolerances)."""
    rng = np.random.default_rng(31)
    x = torch.tensor(rng.standard_normal((4, 70, 6)), dtype=dtype)
    y = torch.tensor(rng.standard_normal((4, 55, 6)), dtype=dtype)
    xd = x.cuda().requires_grad_(True)
    yd = y.cuda().requires_grad_(True)
    out = SoftDTW(gamma=1.0, fused=fused)(xd, yd)
    assert out.dtype == dtype
    out.sum().backward()
    torch.cuda.synchronize()
    _native.check_status()
    assert xd.grad.dtype == dtype and yd.grad.dtype == dtype
    xr, yr = x.float().numpy(), y.float().numpy()
    o64, gx64, gy64 = O.loss_and_grads(xr, yr, gamma=1.0, fused=fused, precision="float64")
    _, gx32, gy32 = O.loss_and_grads(xr, yr, gamma=1.0, fused=fused)
    ulp = {torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8}[dtype]
    assert_loss_close(out.detach().float().cpu().numpy(), o64, rtol=1e-5 + ulp, what="half-input loss vs float64")
    # As in every gradient check: the reference's own float32 noise floor for
    # this input (the gradient is a difference of two larger terms), plus half
    # an ulp of the output dtype in the relative tolerance.
    for got, ref, r32, what in ((xd.grad, gx64, gx32, "grad_x"), (yd.grad, gy64, gy32, "grad_y")):
        assert_grad_close(got.float().cpu().numpy(), ref, floor=noise_floor(r32, ref), rtol=1e-4 + ulp,
                          what=f"half-input {what} vs float64")
