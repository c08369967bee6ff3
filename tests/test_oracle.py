"""The oracle (oracle/sdtw_oracle.c + oracle/oracle.py) is pinned against the
golden fixtures that the reference itself produced (tests/golden/make_golden.py).

* launcher level (D -> R -> E): bit-exact, every case;
* pipeline level (x, y -> loss, grads): the oracle builds D with numpy instead
  of torch, so D differs by a few ulps; losses agree to 1e-6 and gradients
  within the reference's own float32 noise floor.
"""
import numpy as np
import pytest

from conftest import golden, golden_manifest
from _tol import assert_grad_close, assert_loss_close, noise_floor
from oracle import oracle as O

MAN = golden_manifest()
CASES = [n for n in MAN if not n.startswith("_") and n != "bary"]
TABLE_CASES = [n for n in CASES if MAN[n]["tables"]]


@pytest.mark.parametrize("name", TABLE_CASES)
def test_oracle_forward_backward_bit_exact(name):
    m = MAN[name]
    z = golden(name)
    out, R, _ = O.forward(z["D"], m["gamma"], m["bandwidth"])
    assert R.dtype == z["R"].dtype
    assert np.array_equal(R, z["R"]), "R differs from the reference"
    assert np.array_equal(out, z["R"][:, -2, -2])
    E = O.backward(z["D"], R, m["gamma"], m["bandwidth"])
    assert np.array_equal(E, z["E"]), "E differs from the reference"


@pytest.mark.parametrize("name", CASES)
def test_oracle_pipeline_matches_reference(name):
    m = MAN[name]
    z = golden(name)
    B = z["x"].shape[0]
    g = None if m["reduction"] == "sum" else np.full(B, 1.0 / B)
    prec = "float64" if m["dtype"] == "float64" else "reference"
    kw = dict(gamma=m["gamma"], bandwidth=m["bandwidth"], normalize=m["normalize"], grad_out=g)
    out, gx, gy = O.loss_and_grads(z["x"], z["y"], precision=prec, **kw)
    assert_loss_close(out, z["out"], rtol=1e-6)
    if prec == "float64":
        assert_grad_close(gx, z["grad_x"], rtol=1e-10, atol=1e-12)
        assert_grad_close(gy, z["grad_y"], rtol=1e-10, atol=1e-12)
        return
    _, gx64, gy64 = O.loss_and_grads(z["x"], z["y"], precision="float64", **kw)
    assert_grad_close(gx, z["grad_x"], floor=2 * noise_floor(z["grad_x"], gx64))
    assert_grad_close(gy, z["grad_y"], floor=2 * noise_floor(z["grad_y"], gy64))


def test_oracle_barycenter_inputs_present():
    z = golden("bary")
    assert z["X"].shape == (16, 20, 2) and z["bary"].shape == (20, 2)


def test_sim_fused_kernel_semantics():
    """The reference's CUDA fused kernels (run under the Numba simulator when the
    fixture was made) equal the CPU DP fed the direct-difference cost."""
    z = golden("sim_fused")
    D = O.cost_direct(z["x"], z["y"])
    out, R, R64 = O.forward(D, 1.0)
    fin = np.isfinite(z["R"])
    # The GPU path rounds R to float32 cell by cell; the CPU DP rounds once.
    np.testing.assert_allclose(R[fin], z["R"][fin], rtol=2e-6)
    E = O.backward(D.astype(np.float32), R, 1.0)
    np.testing.assert_allclose(E, z["E"], rtol=1e-3, atol=1e-5)


def test_sim_gpu_bandwidth_divergence_documented():
    """With a band, the reference's GPU backward yields NaN at band edges while
    its CPU backward is finite; the B200 build follows the CPU semantics."""
    z = golden("sim_bw_gpu")
    assert np.isnan(z["E"]).any()
    out, R, _ = O.forward(z["D"], float(z["gamma"]), float(z["bandwidth"]))
    E = O.backward(z["D"], R, float(z["gamma"]), float(z["bandwidth"]))
    assert np.isfinite(E).all()
