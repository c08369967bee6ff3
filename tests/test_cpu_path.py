"""The package's host implementation (CPU tensors) against the reference
fixtures and the float64 oracle; float64 gradients checked by gradcheck."""
import numpy as np
import pytest
import torch

from conftest import golden, golden_manifest
from _tol import assert_grad_close, assert_loss_close, noise_floor
from oracle import oracle as O
from softdtw_cuda import SoftDTW
from softdtw_cuda.cuda import launcher

MAN = golden_manifest()
CASES = [n for n in MAN if not n.startswith("_") and n != "bary"]


def _run(z, m):
    dt = torch.float64 if m["dtype"] == "float64" else torch.float32
    x = torch.tensor(z["x"], dtype=dt, requires_grad=True)
    y = torch.tensor(z["y"], dtype=dt, requires_grad=True)
    out = SoftDTW(gamma=m["gamma"], bandwidth=m["bandwidth"], normalize=m["normalize"], fused=False)(x, y)
    loss = out.sum() if m["reduction"] == "sum" else out.mean()
    loss.backward()
    return out.detach().numpy(), x.grad.numpy(), y.grad.numpy()


@pytest.mark.parametrize("name", CASES)
def test_cpu_path_matches_reference(name):
    m = MAN[name]
    z = golden(name)
    out, gx, gy = _run(z, m)
    assert_loss_close(out, z["out"])
    if m["dtype"] == "float64":
        assert_grad_close(gx, z["grad_x"], rtol=1e-9, atol=1e-11)
        assert_grad_close(gy, z["grad_y"], rtol=1e-9, atol=1e-11)
        return
    B = z["x"].shape[0]
    g = None if m["reduction"] == "sum" else np.full(B, 1.0 / B)
    kw = dict(gamma=m["gamma"], bandwidth=m["bandwidth"], normalize=m["normalize"], grad_out=g)
    _, gx64, gy64 = O.loss_and_grads(z["x"], z["y"], precision="float64", **kw)
    # Against the float64 truth: at least as close as the reference itself.
    assert_grad_close(gx, gx64, floor=noise_floor(z["grad_x"], gx64), what="grad_x vs float64")
    assert_grad_close(gy, gy64, floor=noise_floor(z["grad_y"], gy64), what="grad_y vs float64")
    # Against the reference: within its noise floor.
    assert_grad_close(gx, z["grad_x"], floor=2 * noise_floor(z["grad_x"], gx64), what="grad_x vs reference")
    assert_grad_close(gy, z["grad_y"], floor=2 * noise_floor(z["grad_y"], gy64), what="grad_y vs reference")


@pytest.mark.parametrize("normalize,bw", [(False, None), (True, None), (False, 2.0)])
def test_cpu_gradcheck_float64(normalize, bw):
    torch.manual_seed(0)
    x = torch.randn(2, 6, 2, dtype=torch.float64, requires_grad=True)
    y = torch.randn(2, 6, 2, dtype=torch.float64, requires_grad=True)
    f = SoftDTW(gamma=0.7, normalize=normalize, bandwidth=bw, fused=False)
    assert torch.autograd.gradcheck(lambda a, b: f(a, b), (x, y), eps=1e-6, atol=1e-7, rtol=1e-5)


def test_cpu_launcher_compat_tables():
    """launcher.softdtw_forward_cpu/backward_cpu keep the reference layout."""
    z = golden("c1")
    D = torch.tensor(z["D"])
    out, R = launcher.softdtw_forward_cpu(D, 1.0, -1.0)
    assert R.shape == z["R"].shape and R.dtype == torch.float32
    fin = np.isfinite(z["R"])
    assert np.array_equal(np.isfinite(R.numpy()), fin)
    np.testing.assert_allclose(R.numpy()[fin], z["R"][fin], rtol=1e-7, atol=0)
    E = launcher.softdtw_backward_cpu(D, R, 1.0, -1.0)
    _, R64, _ = O.forward(z["D"].astype(np.float64), 1.0)
    E64 = O.backward(z["D"].astype(np.float64), R64, 1.0)
    np.testing.assert_allclose(E.numpy(), E64, rtol=1e-4, atol=1e-6)


def test_cpu_barycenter_matches_reference():
    from softdtw_cuda import softdtw_barycenter_cpu
    z = golden("bary")
    X = torch.tensor(z["X"])
    b = softdtw_barycenter_cpu(X, gamma=1.0, max_iter=10, lr=0.1, early_stopping=False)
    np.testing.assert_allclose(b.numpy(), z["bary"], rtol=1e-4, atol=1e-5)
    bw = softdtw_barycenter_cpu(X, gamma=1.0, weights=torch.tensor(z["weights"]), max_iter=10, lr=0.1,
                                early_stopping=False)
    np.testing.assert_allclose(bw.numpy(), z["bary_w"], rtol=1e-4, atol=1e-5)
