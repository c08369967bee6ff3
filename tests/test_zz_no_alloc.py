"""The allocation-free forward (sdtw_forward_noalloc_f32), called through the C ABI.

It exists for callers that cannot allocate device memory when they call the
library (an allocator that owns all of device memory, a plugin boundary that
passes only inputs and outputs, a loop where cudaMalloc is not allowed); its
scratch is a fixed device array inside the library.  The result must equal the
workspace-based sdtw_forward_f32 on the same input, call after call, since the
shared array keeps whatever the previous call left in it.

This file is named to be collected last, so a failure here stops a `-x` run
only after every other test has run.
"""
import ctypes
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

from _tol import assert_loss_close
from conftest import PKG, ROOT
from oracle import oracle as O
from softdtw_cuda import _native

pytestmark = pytest.mark.gpu


def _forward_with_workspace(D, gamma, bw):
    out, score = _native.forward(D, gamma, bw)
    torch.cuda.synchronize()
    return out, score


def _forward_noalloc(D, gamma, bw):
    B, N, M = D.shape
    L = _native.lib()
    score = torch.empty(_native.score_elems(B, N, M), dtype=torch.float32, device=D.device)
    out = torch.empty(B, dtype=torch.float32, device=D.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(D.device).cuda_stream)
    rc = L.sdtw_forward_noalloc_f32(ctypes.c_void_p(D.data_ptr()), ctypes.c_void_p(score.data_ptr()),
                                    ctypes.c_void_p(out.data_ptr()), B, N, M, float(gamma), float(bw), stream)
    assert rc == 0, L.sdtw_last_error_message().decode()
    torch.cuda.synchronize()
    assert _native.status() == 0
    return out, score


@pytest.mark.parametrize("shape,gamma,bw", [((4, 64, 64), 1.0, -1.0), ((3, 100, 77), 0.1, -1.0),
                                            ((2, 300, 280), 1.0, 30.0)])
def test_noalloc_matches_workspace_forward_twice(shape, gamma, bw):
    B, N, M = shape
    torch.manual_seed(0)
    D1 = torch.rand(B, N, M, device="cuda") * 3.0
    D2 = torch.rand(B, N, M, device="cuda") * 3.0
    for D in (D1, D2):  # two calls in a row, with different inputs
        ref_out, ref_score = _forward_with_workspace(D, gamma, bw)
        out, score = _forward_noalloc(D, gamma, bw)
        # Same kernels on the same input: bit-identical (tolerance 0 leaves room
        # for nothing; the rtol below is the tests' loss tolerance, as a bound).
        np.testing.assert_allclose(out.cpu().numpy(), ref_out.cpu().numpy(), rtol=1e-5, atol=0)
        assert torch.equal(out, ref_out)
        assert torch.equal(score, ref_score)


def test_noalloc_long_problem_uses_the_band_ring():
    """Few warps per band force several bands: the band-wrap ring in the fixed
    array must be reset between calls (it keeps the previous call's tags)."""
    torch.manual_seed(1)
    D = torch.rand(1, 700, 650, device="cuda")
    _native.set_plan_override(2, 2, 1)
    try:
        ref_out, _ = _forward_with_workspace(D, 1.0, -1.0)
        a, _ = _forward_noalloc(D, 1.0, -1.0)
        b, _ = _forward_noalloc(D, 1.0, -1.0)
    finally:
        _native.set_plan_override(0, 0, 0)
    assert torch.equal(a, ref_out) and torch.equal(b, ref_out)


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    L = _native.lib()
    D = torch.zeros(1, 1, 1, device="cuda")  # never read: the size check comes first
    rc = L.sdtw_forward_noalloc_f32(ctypes.c_void_p(D.data_ptr()), ctypes.c_void_p(D.data_ptr()),
                                    ctypes.c_void_p(D.data_ptr()), 64, 1024, 1024, 1.0, -1.0, None)
    assert rc == 1
    assert b"too large for the allocation-free forward" in L.sdtw_last_error_message()


def test_noalloc_matches_oracle():
    """The allocation-free forward against the reference's CPU algorithm (the
    oracle) on a seeded cost matrix, at the tests' loss tolerance."""
    rng = np.random.default_rng(21)
    Dn = (rng.random((3, 90, 70)) * 4.0).astype(np.float32)
    D = torch.tensor(Dn, device="cuda")
    for gamma in (0.1, 1.0):
        out, _ = _forward_noalloc(D, gamma, -1.0)
        ref, _, _ = O.forward(Dn, gamma)
        assert_loss_close(out.cpu().numpy(), ref, what=f"no-alloc forward vs reference (gamma {gamma})")


_FRESH = textwrap.dedent("""
    import ctypes, sys
    sys.path[:0] = [{root!r}, {pkg!r}]
    import numpy as np, torch
    from oracle import oracle as O
    from softdtw_cuda import _native

    L = _native.lib()
    rng = np.random.default_rng(5)
    Dn = (rng.random((1, 64, 64)) * 2.0).astype(np.float32)  # two 32-row stripes
    D = torch.tensor(Dn, device="cuda")
    score = torch.empty(_native.score_elems(1, 64, 64), dtype=torch.float32, device="cuda")
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call():
        return L.sdtw_forward_noalloc_f32(ctypes.c_void_p(D.data_ptr()), ctypes.c_void_p(score.data_ptr()),
                                          ctypes.c_void_p(out.data_ptr()), 1, 64, 64, 1.0, -1.0, st)

    # The first library call of the process: stripe 0 withholds its rows, so
    # stripe 1's bounded wait runs out after 0.2 s.
    L.sdtw_set_wait_timeout_ns(200000000)
    L.sdtw_debug_stall_stripe(0)
    assert call() == 0, L.sdtw_last_error_message()
    torch.cuda.synchronize()
    rc = L.sdtw_status()
    msg = L.sdtw_last_error_message().decode()
    assert rc == 3, (rc, msg)
    assert "allocation-free" in msg and "wait" in msg, msg
    assert L.sdtw_status() == 0  # read and cleared
    L.sdtw_debug_stall_stripe(-1)
    L.sdtw_set_wait_timeout_ns(2000000000)
    ref = O.forward(Dn, 1.0)[0]
    # The context and the library keep working: the same entry point, then the
    # workspace forward, both exact against the oracle.
    assert call() == 0, L.sdtw_last_error_message()
    torch.cuda.synchronize()
    assert L.sdtw_status() == 0
    a = out.cpu().numpy()
    b = _native.forward(D, 1.0, -1.0)[0].cpu().numpy()
    torch.cuda.synchronize()
    assert L.sdtw_status() == 0
    for v in (a, b):
        assert np.max(np.abs(v - ref) / np.abs(ref)) <= 1e-5, (v, ref)
    print("fresh-process no-alloc timeout ok")
""")


def test_noalloc_first_call_timeout_is_reported():
    """Failure detection when the allocation-free forward is the first and only
    library call of a process (so the mapped host status record of the other
    entry points does not exist): a withheld stripe makes a bounded wait run
    out, sdtw_status() reports it after the caller synchronises, and later
    calls are exact.  Runs in a fresh interpreter; no GPU fault is involved."""
    code = _FRESH.format(root=ROOT, pkg=PKG)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "fresh-process no-alloc timeout ok" in r.stdout
