"""Argument validation: same exception types and messages as the reference
(softdtw_cuda/tests/test_validation.py, module.py:35-38, 73-94, checks.py:6-15)."""
import math

import pytest
import torch

from softdtw_cuda import SoftDTW, softdtw
from softdtw_cuda.autograd import SoftDTWAutograd
from softdtw_cuda.distances import pairwise_distance, sqeuclidean
from softdtw_cuda.utils.checks import check_D


@pytest.mark.parametrize("g", [0.0, -1.0])
def test_gamma_nonpositive_raises(g):
    with pytest.raises(ValueError, match="gamma must be > 0"):
        SoftDTW(gamma=g)


@pytest.mark.parametrize("g", [math.inf, math.nan])
def test_gamma_nonfinite_raises(g):
    with pytest.raises(ValueError, match="gamma must be finite"):
        SoftDTW(gamma=g)


def test_fused_true_on_cpu_raises():
    with pytest.raises(ValueError, match="fused=True requires CUDA"):
        SoftDTW(gamma=1.0, fused=True)(torch.randn(2, 5, 3), torch.randn(2, 5, 3))


def test_normalize_unequal_lengths_raises():
    with pytest.raises(ValueError, match="normalize=True"):
        SoftDTW(gamma=1.0, normalize=True)(torch.randn(2, 5, 3), torch.randn(2, 7, 3))


@pytest.mark.parametrize("shapes", [((2, 0, 3), (2, 5, 3)), ((2, 5, 3), (2, 0, 3))])
def test_empty_sequence_raises(shapes):
    with pytest.raises(ValueError, match="Sequence lengths must be > 0"):
        SoftDTW(gamma=1.0)(torch.randn(*shapes[0]), torch.randn(*shapes[1]))


def test_batch_size_mismatch_raises():
    with pytest.raises(ValueError, match="Batch sizes must match"):
        SoftDTW(gamma=1.0)(torch.randn(2, 5, 3), torch.randn(3, 5, 3))


def test_feature_dim_mismatch_raises():
    with pytest.raises(ValueError, match="Feature dims must match"):
        SoftDTW(gamma=1.0)(torch.randn(2, 5, 3), torch.randn(2, 5, 4))


def test_bad_rank_raises():
    with pytest.raises(ValueError, match="Expected x,y to have shape"):
        SoftDTW()(torch.randn(2, 2, 5, 3), torch.randn(2, 5, 3))


def test_unknown_dist_raises():
    with pytest.raises(ValueError, match="Unknown dist"):
        pairwise_distance(torch.randn(1, 3, 2), torch.randn(1, 3, 2), dist="cosine")


def test_sqeuclidean_shape_errors():
    with pytest.raises(ValueError, match="Expected x,y as"):
        sqeuclidean(torch.randn(3, 2), torch.randn(1, 3, 2))
    with pytest.raises(ValueError, match="Batch/features mismatch"):
        sqeuclidean(torch.randn(1, 3, 2), torch.randn(1, 3, 4))


def test_check_D():
    with pytest.raises(TypeError, match="D must be a torch.Tensor"):
        check_D([[1.0]])
    with pytest.raises(ValueError, match="D must have shape"):
        check_D(torch.zeros(3, 3))
    with pytest.raises(TypeError, match="Unsupported dtype"):
        check_D(torch.zeros(1, 3, 3, dtype=torch.int32))
    check_D(torch.zeros(1, 3, 3).transpose(1, 2))  # non-contiguous is accepted


def test_autograd_gamma_check():
    with pytest.raises(ValueError, match="gamma must be > 0"):
        SoftDTWAutograd.apply(torch.rand(1, 3, 3), 0.0, None)


def test_bandwidth_nonpositive_disables():
    assert SoftDTW(bandwidth=0).bandwidth is None
    assert SoftDTW(bandwidth=-3).bandwidth is None
    assert SoftDTW(bandwidth=2).bandwidth == 2.0


def test_functional_fused_none_runs_on_cpu():
    torch.manual_seed(0)
    out = softdtw(torch.randn(2, 5, 3), torch.randn(2, 5, 3), fused=None)
    assert out.shape == (2,) and torch.isfinite(out).all()


def test_unbatched_inputs():
    torch.manual_seed(0)
    out = softdtw(torch.randn(7, 3), torch.randn(5, 3))
    assert out.shape == (1,)


def test_normalize_bindings_check_their_pair():
    """The in-place normalize bindings refuse mismatched or host tensors
    before calling the library."""
    from softdtw_cuda import _native
    x = torch.zeros(2, 5, 3)
    with pytest.raises(ValueError, match="normalize"):
        _native.forward_xy_norm(x, x, 1.0, -1.0)
    with pytest.raises(ValueError, match="normalize"):
        _native.forward_sqeuclid_norm(x, torch.zeros(2, 4, 3), 1.0, -1.0)
