"""dL/dx alone (y constant): the reverse pass applies the chain rule itself
(no E table, no gradient kernel).  Its dL/dx must equal the one computed with
both gradients (E table + gradient kernel), on many shapes and launch
geometries, including multi-band plans."""
import pytest
import torch

from softdtw_cuda import SoftDTW, _native

pytestmark = pytest.mark.gpu


def _grads(x, y, gamma, need_y):
    xr = x.clone().requires_grad_(True)
    yr = y.clone().requires_grad_(need_y)
    w = torch.linspace(0.5, 1.5, x.shape[0], device=x.device)
    (w * SoftDTW(gamma=gamma, fused=True)(xr, yr)).sum().backward()
    return xr.grad


@pytest.mark.parametrize("B,N,M,D", [(4, 100, 100, 3), (3, 33, 70, 8), (2, 65, 40, 16), (5, 1, 9, 2), (2, 130, 7, 4),
                                     (3, 64, 64, 12)])
@pytest.mark.parametrize("plan", [None, (2, 1, 1), (4, 2, 1)])
def test_gradx_only_matches_both(B, N, M, D, plan):
    g = torch.Generator().manual_seed(B * 100 + N + D)
    x = torch.randn(B, N, D, generator=g).cuda()
    y = torch.randn(B, M, D, generator=g).cuda()
    if plan:
        _native.set_plan_override(*plan)
    try:
        gx_only = _grads(x, y, 0.5, False)
        gx_both = _grads(x, y, 0.5, True)
    finally:
        _native.set_plan_override(0, 0, 0)
    torch.cuda.synchronize()
    scale = gx_both.abs().max().item()
    torch.testing.assert_close(gx_only, gx_both, rtol=1e-4, atol=1e-5 * max(scale, 1.0))
