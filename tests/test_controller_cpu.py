"""Host logic of the controller scalars against the oracle (no GPU): the shrinkage-RLOO
advantages and reward EMA (ds_mezo/controller.py:216-229) over a run of steps, the eps
median rule (ds_mezo/controller.py:78-82), and the skipped-step rule (:299-301)."""
import math

import torch

from oracle import reference_ops as ref


def test_shrinkage_rloo_matches_oracle_over_steps():
    from dsmezo_b200 import ShrinkageRLOO
    g = torch.Generator().manual_seed(3)
    ours = ShrinkageRLOO()
    ema = 0.0
    for step in range(1, 9):
        rewards = (torch.rand(4, generator=g) * 2 - 0.5).tolist()
        if step == 3:
            rewards = [1.0, 1.0, 1.0, 1.0]            # zero variance: lam = 0
        momentum = 0.0 if step == 1 else 1.0 - 1.0 / min(step - 1, 10)
        want, ema = ref.shrinkage_rloo(rewards, ema, momentum)
        got = ours.advantages(rewards, momentum)
        assert got == want, (step, got, want)
        assert ours.reward_ema == ema


def test_controller_advantages_use_the_previous_momentum():
    from dsmezo_b200 import ShrinkageRLOO
    from dsmezo_b200.adapter_set import kalman_beta_q
    # the reference's _explore at step s uses the momentum _update_weights set at step s-1
    r = ShrinkageRLOO()
    ema = 0.0
    for s in range(1, 5):
        prev_beta = 0.0 if s == 1 else kalman_beta_q(s - 1, 100, 1e-3)[0]
        rewards = [0.1 * s, 0.5, -0.2, 0.3 * s]
        want, ema = ref.shrinkage_rloo(rewards, ema, prev_beta)
        assert r.advantages(rewards, prev_beta) == want


def test_eps_median_rule():
    from dsmezo_b200 import eps_from_norms
    norms = torch.tensor([5.0, 1.0, 3.0, 2.0, 4.0, 6.0])
    # torch.median of an even count is the lower middle value (3.0 here, not 3.5)
    assert float(torch.median(norms)) == 3.0
    assert math.isclose(eps_from_norms(norms), 3.0 * float(torch.finfo(torch.float32).eps) ** (1 / 3), rel_tol=0)
    A = [torch.randn(7, 3, generator=torch.Generator().manual_seed(i)) for i in range(5)]
    B = [torch.randn(3, 9, generator=torch.Generator().manual_seed(10 + i)) for i in range(5)]
    n = torch.tensor([float(torch.linalg.norm(a)) for a in A] + [float(torch.linalg.norm(b)) for b in B])
    assert eps_from_norms(n) == ref.eps_from_factors(A, B)
