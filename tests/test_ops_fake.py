"""The torch.compile custom operators (softdtw_cuda/ops.py) without a GPU:
registration and the fake (meta) implementations' shapes and dtypes."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import softdtw_cuda  # noqa: F401  (registers the operators)
from softdtw_cuda import _native


def test_operators_registered():
    for name in ("xy_forward", "xy_backward", "sq_forward", "sq_backward", "d_forward", "d_backward"):
        assert hasattr(torch.ops.softdtw_cuda, name), name


def test_fake_shapes():
    B, N, M, Dm = 3, 40, 33, 5
    with FakeTensorMode():
        x = torch.empty(B, N, Dm, device="cuda", dtype=torch.bfloat16)
        y = torch.empty(B, M, Dm, device="cuda", dtype=torch.bfloat16)
        out, score = torch.ops.softdtw_cuda.xy_forward(x, y, 1.0, -1.0)
        assert out.shape == (B,) and out.dtype == torch.bfloat16
        assert score.shape == (_native.score_elems(B, N, M),) and score.dtype == torch.float32
        g = torch.empty(B, device="cuda", dtype=torch.bfloat16)
        gx, gy = torch.ops.softdtw_cuda.xy_backward(x, y, score, g, 1.0, -1.0, True, False)
        assert gx.shape == x.shape and gx.dtype == x.dtype and gy.numel() == 0
        out, score, cost = torch.ops.softdtw_cuda.sq_forward(x, y, 0.5, 3.0)
        assert cost.shape == (_native.cost_elems(B, N, M),)
        D = torch.empty(B, N, M, device="cuda")
        out, score = torch.ops.softdtw_cuda.d_forward(D, 1.0, -1.0)
        E = torch.ops.softdtw_cuda.d_backward(score, out, B, N, M, 1.0, -1.0)
        assert E.shape == (B, N, M)
