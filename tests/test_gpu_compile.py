"""SoftDTW under torch.compile: the custom operators (softdtw_cuda/ops.py) pass
torch.library.opcheck, and a compiled training step (fullgraph, no graph break
at the loss) gives the eager step's loss and gradients."""
import pytest
import torch

from softdtw_cuda import SoftDTW

pytestmark = pytest.mark.gpu


def _xy(seed, B=3, N=24, M=19, Dm=4, dtype=torch.float32):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, N, Dm, device="cuda", dtype=dtype, generator=g, requires_grad=True)
    y = torch.randn(B, M, Dm, device="cuda", dtype=dtype, generator=g, requires_grad=True)
    return x, y


def test_opcheck():
    x, y = _xy(0)
    g = torch.rand(3, device="cuda")
    torch.library.opcheck(torch.ops.softdtw_cuda.xy_forward, (x, y, 1.0, -1.0))
    # sq_forward's cost table leaves the wavefront layout's padding cells
    # unwritten (nothing reads them), so two runs differ there: its output
    # comparison under AOT dispatch is skipped; schema, fake and autograd
    # registration are still checked.
    torch.library.opcheck(torch.ops.softdtw_cuda.sq_forward, (x, y, 0.5, 4.0),
                          test_utils=("test_schema", "test_autograd_registration", "test_faketensor"))
    out, score = torch.ops.softdtw_cuda.xy_forward(x.detach(), y.detach(), 1.0, -1.0)
    torch.library.opcheck(torch.ops.softdtw_cuda.xy_backward,
                          (x.detach(), y.detach(), score, g, 1.0, -1.0, True, True))
    D = torch.rand(2, 9, 7, device="cuda", requires_grad=True)
    torch.library.opcheck(torch.ops.softdtw_cuda.d_forward, (D, 1.0, -1.0))


class _Model(torch.nn.Module):
    def __init__(self, fused, normalize=False):
        super().__init__()
        self.proj = torch.nn.Linear(4, 4)
        self.loss = SoftDTW(gamma=0.5, fused=fused, normalize=normalize)

    def forward(self, x, y):
        return self.loss(self.proj(x), y).mean()


@pytest.mark.parametrize("fused,normalize,backend", [(True, False, "aot_eager"), (False, False, "aot_eager"),
                                                     (True, True, "aot_eager"), (True, False, "inductor")])
def test_compiled_step_matches_eager(fused, normalize, backend):
    torch.manual_seed(0)
    model = _Model(fused, normalize).cuda()
    N = M = 21 if normalize else None
    x, y = _xy(1, N=N or 24, M=M or 19)
    eager = model(x, y)
    ge = torch.autograd.grad(eager, (x, y, model.proj.weight))
    compiled = torch.compile(model, fullgraph=True, backend=backend)
    c = compiled(x, y)
    gc = torch.autograd.grad(c, (x, y, model.proj.weight))
    torch.testing.assert_close(c, eager, rtol=1e-6, atol=1e-6)
    for u, v in zip(gc, ge):
        torch.testing.assert_close(u, v, rtol=1e-5, atol=1e-6)
