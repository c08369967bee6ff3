"""GPU parity: the libsdtw_b200 kernels against the reference fixtures and the
oracle (reference CPU algorithm, float32 and float64), on seeded inputs.

Tolerances (see conftest.py): loss 1e-5 relative; gradients rtol 1e-4 /
atol 1e-6 plus the reference's own float32 noise floor for the same input.
"""
import numpy as np
import pytest
import torch

from conftest import golden, golden_manifest
from _tol import assert_grad_close, assert_loss_close, noise_floor
from oracle import oracle as O
from softdtw_cuda import SoftDTW, _native
from softdtw_cuda.cuda import launcher

pytestmark = pytest.mark.gpu

MAN = golden_manifest()
F32_CASES = [n for n in MAN if not n.startswith("_") and n != "bary" and MAN[n]["dtype"] == "float32"]


def _gpu_run(x, y, *, gamma, bandwidth=None, normalize=False, fused=False, reduction="sum"):
    xt = torch.tensor(x, device="cuda", requires_grad=True)
    yt = torch.tensor(y, device="cuda", requires_grad=True)
    out = SoftDTW(gamma=gamma, bandwidth=bandwidth, normalize=normalize, fused=fused)(xt, yt)
    loss = out.sum() if reduction == "sum" else out.mean()
    loss.backward()
    torch.cuda.synchronize()
    _native.check_status()
    return out.detach().cpu().numpy(), xt.grad.cpu().numpy(), yt.grad.cpu().numpy()


def _check_against_oracle(x, y, out, gx, gy, *, gamma, bandwidth=None, normalize=False, fused=False,
                          grad_out=None, ref=None):
    kw = dict(gamma=gamma, bandwidth=bandwidth, normalize=normalize, fused=fused, grad_out=grad_out)
    o32, gx32, gy32 = O.loss_and_grads(x, y, **kw) if ref is None else ref
    o64, gx64, gy64 = O.loss_and_grads(x, y, precision="float64", **kw)
    assert_loss_close(out, o32, what="loss vs reference")
    assert_loss_close(out, o64, what="loss vs float64")
    fx, fy = noise_floor(gx32, gx64), noise_floor(gy32, gy64)
    assert_grad_close(gx, gx64, floor=fx, what="grad_x vs float64")
    assert_grad_close(gy, gy64, floor=fy, what="grad_y vs float64")
    assert_grad_close(gx, gx32, floor=2 * fx, what="grad_x vs reference")
    assert_grad_close(gy, gy32, floor=2 * fy, what="grad_y vs reference")


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("name", F32_CASES)
def test_golden_cases(name, fused):
    m = MAN[name]
    z = golden(name)
    out, gx, gy = _gpu_run(z["x"], z["y"], gamma=m["gamma"], bandwidth=m["bandwidth"], normalize=m["normalize"],
                           fused=fused, reduction=m["reduction"])
    B = z["x"].shape[0]
    g = None if m["reduction"] == "sum" else np.full(B, 1.0 / B)
    if fused:
        # The fused cost is the direct difference (kernels.py:27-31); the fixture
        # used the expanded unfused cost, so compare with the oracle's fused mode.
        _check_against_oracle(z["x"], z["y"], out, gx, gy, gamma=m["gamma"], bandwidth=m["bandwidth"],
                              normalize=m["normalize"], fused=True, grad_out=g)
    else:
        _check_against_oracle(z["x"], z["y"], out, gx, gy, gamma=m["gamma"], bandwidth=m["bandwidth"],
                              normalize=m["normalize"], grad_out=g,
                              ref=(z["out"], z["grad_x"], z["grad_y"]))


@pytest.mark.parametrize("name", [n for n in F32_CASES if MAN[n]["tables"]])
def test_launcher_level_tables(name):
    """D -> R -> E through the reference-layout launcher functions."""
    m = MAN[name]
    z = golden(name)
    D = torch.tensor(z["D"], device="cuda")
    bw = -1.0 if m["bandwidth"] is None else float(m["bandwidth"])
    out, R = launcher.softdtw_forward_cuda(D, m["gamma"], bw)
    Rn = R.cpu().numpy()
    fin = np.isfinite(z["R"])
    assert np.array_equal(np.isfinite(Rn), fin)
    # R accumulates float32 rounding along the path: absolute error ~ |R|max * 1e-6.
    np.testing.assert_allclose(Rn[fin], z["R"][fin], rtol=2e-6, atol=2e-6 * np.abs(z["R"][fin]).max())
    E = launcher.softdtw_backward_cuda_log(D, R, m["gamma"], bw).cpu().numpy()
    _, R64, _ = O.forward(z["D"].astype(np.float64), m["gamma"], m["bandwidth"])
    E64 = O.backward(z["D"].astype(np.float64), R64, m["gamma"], m["bandwidth"])
    floor = noise_floor(z["E"], E64)
    assert_grad_close(E, E64, floor=floor + 1e-5, what="E vs float64")
    assert_grad_close(E, z["E"], floor=2 * floor + 1e-5, what="E vs reference")


SHAPES = [
    (1, 1, 1, 1), (2, 1, 9, 2), (2, 9, 1, 2), (3, 31, 33, 3), (2, 32, 32, 4), (2, 33, 65, 2),
    (5, 64, 17, 3), (1, 100, 100, 8), (3, 129, 200, 5), (40, 70, 70, 3), (2, 300, 257, 6), (1, 513, 511, 3),
]


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_shapes_vs_oracle(shape, fused):
    B, N, M, Dm = shape
    rng = np.random.default_rng(N * 1000 + M)
    x = rng.standard_normal((B, N, Dm)).astype(np.float32)
    y = rng.standard_normal((B, M, Dm)).astype(np.float32)
    out, gx, gy = _gpu_run(x, y, gamma=1.0, fused=fused)
    _check_against_oracle(x, y, out, gx, gy, gamma=1.0, fused=fused)


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("dim", [1, 33, 128, 241, 300, 513])
@pytest.mark.parametrize("NM", [(70, 90), (150, 190)], ids=["rm", "wl"])
def test_feature_dims(dim, fused, NM):
    """Gradients on the tensor cores (3xTF32): feature blocks of up to 240
    columns plus the row-sum column, partial 128-row tiles and K chunks.
    Lengths of at most 128 take the row-major operand kernel, longer ones the
    kernel that reads E from the wavefront layout."""
    rng = np.random.default_rng(dim)
    x = (rng.standard_normal((2, NM[0], dim)) / np.sqrt(dim)).astype(np.float32)
    y = (rng.standard_normal((2, NM[1], dim)) / np.sqrt(dim)).astype(np.float32)
    out, gx, gy = _gpu_run(x, y, gamma=1.0, fused=fused)
    _check_against_oracle(x, y, out, gx, gy, gamma=1.0, fused=fused)


@pytest.mark.parametrize("gamma", [0.01, 0.1, 1.0, 10.0])
@pytest.mark.parametrize("fused", [False, True])
def test_gamma_sweep_mid(gamma, fused):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((8, 256, 16)).astype(np.float32)
    y = rng.standard_normal((8, 256, 16)).astype(np.float32)
    out, gx, gy = _gpu_run(x, y, gamma=gamma, fused=fused)
    _check_against_oracle(x, y, out, gx, gy, gamma=gamma, fused=fused)


@pytest.mark.parametrize("bw", [1.0, 2.5, 10.0, 200.0])
def test_bandwidth(bw):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((3, 90, 4)).astype(np.float32)
    y = rng.standard_normal((3, 80, 4)).astype(np.float32)
    for fused in (False, True):
        out, gx, gy = _gpu_run(x, y, gamma=0.5, bandwidth=bw, fused=fused)
        if bw < 10.0:  # |N - M| = 10 > bw: the corner is outside the band
            assert np.isinf(out).all() and np.all(gx == 0) and np.all(gy == 0)
        _check_against_oracle(x, y, out, gx, gy, gamma=0.5, bandwidth=bw, fused=fused)


def test_normalize_fused_matches_unfused():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((4, 60, 3)).astype(np.float32)
    y = rng.standard_normal((4, 60, 3)).astype(np.float32)
    for fused in (False, True):
        out, gx, gy = _gpu_run(x, y, gamma=1.0, normalize=True, fused=fused)
        _check_against_oracle(x, y, out, gx, gy, gamma=1.0, normalize=True, fused=fused)


def test_headline_shape_c2():
    """BASELINE config 2 at full size (B=32, N=M=512, D=64), fused and unfused,
    mean reduction, against the oracle."""
    torch.manual_seed(0)
    x = torch.randn(32, 512, 64).numpy()
    y = torch.randn(32, 512, 64).numpy()
    g = np.full(32, 1.0 / 32)
    for fused in (False, True):
        out, gx, gy = _gpu_run(x, y, gamma=1.0, fused=fused, reduction="mean")
        _check_against_oracle(x, y, out, gx, gy, gamma=1.0, fused=fused, grad_out=g)


def test_long_multiband_vs_oracle():
    """N = M = 5000 needs two bands of stripes (the band-wrap ring); one problem
    is checked against the oracle."""
    rng = np.random.default_rng(11)
    x = rng.standard_normal((1, 5000, 2)).astype(np.float32)
    y = rng.standard_normal((1, 5000, 2)).astype(np.float32)
    out, gx, gy = _gpu_run(x, y, gamma=1.0, fused=True)
    assert np.isfinite(out).all() and np.isfinite(gx).all() and np.abs(gx).mean() > 0
    _check_against_oracle(x, y, out, gx, gy, gamma=1.0, fused=True)


@pytest.mark.parametrize("wpc,cs,k", [(1, 1, 1), (1, 2, 1), (2, 1, 1), (3, 2, 1), (1, 8, 1), (2, 4, 1),
                                      (1, 1, 2), (2, 2, 2), (1, 1, 4), (1, 2, 4)])
def test_forced_plans_many_bands(wpc, cs, k):
    """Small problems on forced launch geometries: many bands (band-wrap ring),
    every cluster size, stripes split across CTAs, 1/2/4 DP rows per lane;
    fused and unfused."""
    rng = np.random.default_rng(wpc * 10 + cs + 100 * k)
    x = rng.standard_normal((3, 230, 3)).astype(np.float32)
    y = rng.standard_normal((3, 170, 3)).astype(np.float32)
    _native.set_plan_override(wpc, cs, k)
    try:
        for fused in (False, True):
            out, gx, gy = _gpu_run(x, y, gamma=0.5, fused=fused)
            _check_against_oracle(x, y, out, gx, gy, gamma=0.5, fused=fused)
    finally:
        _native.set_plan_override(0, 0)


def test_reference_long_and_small_gamma_smoke():
    """The reference's own finiteness tests (test_softdtw_long.py, test_softdtw_log_backward.py)."""
    torch.manual_seed(0)
    x = torch.randn(2, 128, 3, device="cuda", requires_grad=True)
    y = torch.randn(2, 128, 3, device="cuda")
    out = SoftDTW(gamma=0.01)(x, y)
    out.sum().backward()
    assert torch.isfinite(out).all() and torch.isfinite(x.grad).all() and x.grad.abs().mean() > 1e-6


def test_deterministic():
    torch.manual_seed(1)
    x = torch.randn(6, 200, 8, device="cuda")
    y = torch.randn(6, 180, 8, device="cuda")
    res = []
    for _ in range(2):
        xr = x.clone().requires_grad_(True)
        o = SoftDTW(gamma=0.3)(xr, y)
        o.sum().backward()
        res.append((o.detach().clone(), xr.grad.clone()))
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])


def test_side_stream_and_half_inputs():
    torch.manual_seed(2)
    x = torch.randn(3, 50, 4, device="cuda")
    y = torch.randn(3, 40, 4, device="cuda")
    ref = SoftDTW()(x, y)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        o = SoftDTW()(x, y)
    s.synchronize()
    assert torch.equal(o, ref)
    oh = SoftDTW(fused=False)(x.half(), y.half())
    assert oh.dtype == torch.float16 and torch.isfinite(oh).all()


def test_wait_timeout_reports_and_context_survives():
    """Failure detection without a fault: the producer of stripe 1 withholds its
    rows, the consumer's bounded wait runs out, the status word reports it, the
    host raises, and the context keeps working."""
    x = torch.randn(1, 64, 3, device="cuda")
    y = torch.randn(1, 64, 3, device="cuda")
    good = SoftDTW(fused=False)(x, y)
    torch.cuda.synchronize()
    _native.set_wait_timeout(0.2)
    _native.debug_stall_stripe(0)
    try:
        SoftDTW(fused=False)(x, y)
        with pytest.raises(RuntimeError, match="wait"):
            _native.check_status()
    finally:
        _native.debug_stall_stripe(-1)
        _native.set_wait_timeout(2.0)
    again = SoftDTW(fused=False)(x, y)
    _native.check_status()
    assert torch.equal(again, good)
