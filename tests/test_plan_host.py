"""Launch-plan invariants of the library's host code, without a GPU: the
stripe, band and cluster arithmetic of sdtw_plan.h and plan() in capi.cu, and
the plan override the tests use to force many bands and clusters."""
import itertools

import pytest

from softdtw_cuda import _native

SHAPES = [(1, 1, 1), (4, 64, 64), (32, 512, 512), (16, 4096, 4096), (64, 1024, 768), (192, 1024, 1024),
          (4096, 100, 100), (3, 5000, 7), (148, 32, 512)]


def _check(info, N):
    K = info["rows_per_lane"]
    assert K in (1, 2, 4)
    assert info["stripes"] == -(-N // (32 * K))
    assert 1 <= info["warps_per_cta"] <= 8
    assert info["cluster_size"] in (1, 2, 4, 8)
    G = info["warps_per_cta"] * info["cluster_size"]
    assert info["bands"] == -(-info["stripes"] // G)


@pytest.mark.parametrize("B,N,M", SHAPES)
def test_automatic_plan_invariants(B, N, M):
    info = _native.plan_info(B, N, M)
    _check(info, N)
    assert info["rows_per_lane"] == 1
    # The cost table of the unfused pair: one row per lane, n_diag rows per stripe
    # (M + 31 rounded up to 16, plus 16 rows of padding).
    n_diag = (M + 31 + 15) // 16 * 16 + 16
    assert _native.cost_elems(B, N, M) == B * info["stripes"] * n_diag * 32


@pytest.mark.parametrize("w,c,k", list(itertools.product((1, 3, 8), (1, 2, 8), (1, 2, 4))))
def test_plan_override_is_obeyed(w, c, k):
    try:
        _native.set_plan_override(w, c, k)
        info = _native.plan_info(4, 700, 300)
    finally:
        _native.set_plan_override(0, 0, 0)
    _check(info, 700)
    assert (info["warps_per_cta"], info["cluster_size"], info["rows_per_lane"]) == (w, c, k)
    assert _native.plan_info(4, 700, 300)["rows_per_lane"] == 1
