"""Host logic of the replayed barycenter loop (no GPU): the learning-rate
table equals what torch's CosineAnnealingLR gives the step-by-step loop, and the
early-stop rule applied to a loss history stops where the reference loop
(barycenters.py:139-155) breaks."""
import torch

import softdtw_cuda.barycenters as bc


def test_cosine_table_matches_scheduler():
    lrs = bc._cosine_lrs(0.1, 17)
    assert len(lrs) == 18
    p = torch.zeros(1, requires_grad=True)
    opt = torch.optim.Adam([p], lr=0.1)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=17, eta_min=0.1 * 0.1)  # as the loop
    for it in range(17):
        assert lrs[it] == opt.param_groups[0]["lr"]
        opt.step()
        sched.step()
    assert abs(lrs[-1] - 0.01) < 1e-12


def _reference_stop(losses, max_iter, patience, tol):
    # The loop of barycenters.py:139-155, restated over a given loss sequence.
    best, stale = float("inf"), 0
    for it, v in enumerate(losses):
        imp = best - v
        if imp > tol:
            best, stale = v, 0
        else:
            stale += 1
        if stale >= patience and it > max_iter // 2:
            return it
    return None


def test_early_stop_rule():
    g = torch.Generator().manual_seed(0)
    for trial in range(200):
        n = int(torch.randint(8, 60, (1,), generator=g))
        steps = torch.rand(n, generator=g) * (0.05 if trial % 2 else 2.0)
        losses = (10.0 - torch.cumsum(steps, 0)).tolist()
        if trial % 3 == 0:  # plateaus
            k = n // 3
            losses[k:] = [losses[k]] * (n - k)
        patience = int(torch.randint(1, 6, (1,), generator=g))
        tol = float(torch.rand(1, generator=g)) * 0.2
        assert bc._early_stop_at(losses, n, patience, tol) == _reference_stop(losses, n, patience, tol)
    # A loss that never improves stops right after max_iter // 2 once patience ran out.
    assert bc._early_stop_at([1.0] * 20, 20, 3, 1e-3) == 11
