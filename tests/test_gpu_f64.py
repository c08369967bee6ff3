"""The float64 CUDA path against the float64 oracle (launcher.py:307-353 in
double), plus gradcheck on the device and fused == unfused in float64."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from softdtw_cuda import SoftDTW, _native
from softdtw_cuda.autograd import SoftDTWAutograd

pytestmark = pytest.mark.gpu

RTOL = 1e-10  # both sides are double; exp/log differ by an ulp between CUDA and libm


@pytest.mark.parametrize("B,N,M", [(3, 17, 23), (2, 1, 9), (2, 40, 1), (1, 70, 66)])
@pytest.mark.parametrize("gamma", [0.1, 1.0])
@pytest.mark.parametrize("bandwidth", [None, 5.0])
def test_f64_tables_match_oracle(B, N, M, gamma, bandwidth):
    rng = np.random.default_rng(N * 1000 + M)
    D = rng.random((B, N, M)) * 4.0
    out_ref, R_ref, _ = O.forward(D, gamma, bandwidth)
    g = rng.random(B) + 0.5
    E_ref = O.backward(D, R_ref, gamma, bandwidth) * g[:, None, None]
    Dt = torch.tensor(D, device="cuda")
    bw = -1.0 if bandwidth is None else float(bandwidth)
    out, R = _native.forward_f64(Dt, gamma, bw)
    E = _native.backward_f64(Dt, R, torch.tensor(g, device="cuda"), gamma, bw)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), out_ref, rtol=RTOL)
    Rn = R.cpu().numpy()
    fin = np.isfinite(R_ref)
    assert np.array_equal(fin, np.isfinite(Rn))
    np.testing.assert_allclose(Rn[fin], R_ref[fin], rtol=RTOL, atol=1e-12)
    np.testing.assert_allclose(E.cpu().numpy(), E_ref, rtol=RTOL, atol=1e-13)


@pytest.mark.parametrize("fused", [True, False])
def test_f64_module_matches_oracle(fused):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 21, 4))
    y = rng.standard_normal((3, 18, 4))
    xt = torch.tensor(x, device="cuda", requires_grad=True)
    yt = torch.tensor(y, device="cuda", requires_grad=True)
    out = SoftDTW(gamma=0.5, fused=fused)(xt, yt)
    assert out.dtype == torch.float64
    out.sum().backward()
    if fused:
        # The fused cost's direct form in double (kernels.py:27-31), then the
        # float64 reference tables and the chain rule of autograd_xy.py:41-49.
        D = ((x[:, :, None, :] - y[:, None, :, :]) ** 2).sum(-1)
        o, R, _ = O.forward(D, 0.5)
        G = O.backward(D, R, 0.5)
        gx = 2.0 * (x * G.sum(2)[:, :, None] - G @ y)
        gy = 2.0 * (y * G.sum(1)[:, :, None] - np.swapaxes(G, 1, 2) @ x)
    else:
        o, gx, gy = O.loss_and_grads(x, y, gamma=0.5, fused=False, precision="float64")
    np.testing.assert_allclose(out.detach().cpu().numpy(), o, rtol=1e-9)
    np.testing.assert_allclose(xt.grad.cpu().numpy(), gx, rtol=1e-8, atol=1e-10)
    np.testing.assert_allclose(yt.grad.cpu().numpy(), gy, rtol=1e-8, atol=1e-10)


def test_f64_gradcheck_on_device():
    torch.manual_seed(0)
    D = torch.rand(2, 5, 4, dtype=torch.float64, device="cuda", requires_grad=True)
    assert torch.autograd.gradcheck(lambda d: SoftDTWAutograd.apply(d, 0.7, None), (D,))
    x = torch.randn(2, 5, 3, dtype=torch.float64, device="cuda", requires_grad=True)
    y = torch.randn(2, 4, 3, dtype=torch.float64, device="cuda", requires_grad=True)
    for fused in (True, False):
        assert torch.autograd.gradcheck(lambda a, b: SoftDTW(gamma=0.7, fused=fused)(a, b), (x, y))


def test_f64_fused_equals_unfused():
    torch.manual_seed(1)
    x = torch.randn(4, 30, 6, dtype=torch.float64, device="cuda", requires_grad=True)
    y = torch.randn(4, 25, 6, dtype=torch.float64, device="cuda", requires_grad=True)
    a = SoftDTW(gamma=1.0, fused=True)(x, y)
    ga = torch.autograd.grad(a.sum(), (x, y))
    b = SoftDTW(gamma=1.0, fused=False)(x, y)
    gb = torch.autograd.grad(b.sum(), (x, y))
    torch.testing.assert_close(a, b, rtol=1e-10, atol=1e-10)
    for u, v in zip(ga, gb):
        torch.testing.assert_close(u, v, rtol=1e-8, atol=1e-10)


@pytest.mark.parametrize("N,M,dim", [(37, 29, 3), (20, 45, 70)])
def test_f64_chain_rule_kernel(N, M, dim):
    """sdtw_grad_sqeuclid_f64 against numpy in double: N != M, feature counts
    below and above one 32-feature block, either gradient alone."""
    rng = np.random.default_rng(N * M + dim)
    G = rng.random((3, N, M))
    x = rng.standard_normal((3, N, dim))
    y = rng.standard_normal((3, M, dim))
    gx_ref = 2.0 * (x * G.sum(2)[:, :, None] - G @ y)
    gy_ref = 2.0 * (y * G.sum(1)[:, :, None] - np.swapaxes(G, 1, 2) @ x)
    t = lambda a: torch.tensor(a, device="cuda")
    gx, gy = _native.grad_sqeuclid_f64(t(G), t(x), t(y))
    np.testing.assert_allclose(gx.cpu().numpy(), gx_ref, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(gy.cpu().numpy(), gy_ref, rtol=1e-12, atol=1e-12)
    gx_only, none = _native.grad_sqeuclid_f64(t(G), t(x), t(y), True, False)
    assert none is None and torch.equal(gx_only, gx)
