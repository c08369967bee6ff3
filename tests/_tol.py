"""Tolerance helpers shared by the parity tests (see conftest.py for the policy)."""
from __future__ import annotations

import numpy as np

LOSS_RTOL = 1e-5
GRAD_RTOL = 1e-4
GRAD_ATOL = 1e-6


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1e-30)))


def assert_loss_close(ours, ref, rtol=LOSS_RTOL, what="loss"):
    ours = np.asarray(ours, np.float64)
    ref = np.asarray(ref, np.float64)
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(ours), fin), f"{what}: finiteness differs"
    err = rel_err(ours[fin], ref[fin]) if fin.any() else 0.0
    assert err <= rtol, f"{what}: max rel err {err:.3e} > {rtol:.1e}"


def assert_grad_close(ours, ref, floor=0.0, rtol=GRAD_RTOL, atol=GRAD_ATOL, what="grad"):
    """|ours - ref| <= rtol*|ref| + atol + floor, elementwise.

    `floor` is the reference's own float32 noise for this input (see
    noise_floor); pass 0 to demand the plain rtol/atol bar."""
    ours = np.asarray(ours, np.float64)
    ref = np.asarray(ref, np.float64)
    bound = rtol * np.abs(ref) + atol + floor
    diff = np.abs(ours - ref)
    bad = diff > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{bad.size} elements outside tolerance; "
                           f"worst diff {diff.max():.3e} (floor {floor:.3e}, scale {np.abs(ref).max():.3e})")


def noise_floor(ref32, ref64):
    """Largest |float32 reference - float64 reference| (the reference's own error)."""
    return float(np.max(np.abs(np.asarray(ref32, np.float64) - np.asarray(ref64, np.float64))))
