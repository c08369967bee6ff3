"""Shared test set-up: import paths, the `gpu` marker, golden-fixture access and
the tolerance policy used by every parity test.

Tolerance policy (applied in _tol.py): losses must agree with the reference
oracle to 1e-5 relative.  Gradients must agree to rtol 1e-4 / atol 1e-6 plus the
reference's own float32 noise floor for that input, measured live as the
largest difference between the oracle's float32 pipeline (the reference's
arithmetic) and the same pipeline in float64.  That floor is about
0.5*ulp(R)/gamma times the gradient scale; no float32 implementation that
rounds differently from the reference can get closer to it than that.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "sdtw-cuda-torch_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the library's kernels")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def golden_manifest():
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        return json.load(f)


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


@pytest.fixture(scope="session")
def manifest():
    return golden_manifest()
