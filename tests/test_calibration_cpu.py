"""Host side of the first-step calibration (ds_mezo/controller.py:135-163): the optht rank
rule against the oracle's independent restatement and the paper's published values, the
oracle's svd_lowrank restatement against torch.svd_lowrank itself (same sketch), and the
rank median over ranks (gloo, world size 2)."""
import math
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import reference_ops as ref


@pytest.mark.parametrize("beta", [1.0, 0.999, 0.75, 0.5, 0.25, 0.1, 0.01, 1e-3])
def test_mp_median_closed_form_matches_quadrature(beta):
    from dsmezo_b200.calibration import marchenko_pastur_median
    assert math.isclose(marchenko_pastur_median(beta), ref.mp_median_quadrature(beta), rel_tol=1e-11)


def test_threshold_published_values():
    """Gavish & Donoho 2014: lambda*(1) = 4/sqrt(3), omega(1) ~= 2.858, and the cubic fit
    omega(beta) ~= 0.56 b^3 - 0.95 b^2 + 1.82 b + 1.43 to about 0.02 on [0.01, 1]."""
    from dsmezo_b200.calibration import optimal_threshold_coefficient, optimal_threshold_known_noise
    assert math.isclose(optimal_threshold_known_noise(1.0), 4.0 / math.sqrt(3.0), rel_tol=1e-15)
    assert abs(optimal_threshold_coefficient(1.0) - 2.858) < 1e-3
    for beta in np.linspace(0.01, 1.0, 34):
        fit = 0.56 * beta ** 3 - 0.95 * beta ** 2 + 1.82 * beta + 1.43
        assert abs(optimal_threshold_coefficient(float(beta)) - fit) < 0.02


@pytest.mark.parametrize("shape,k,seed", [((400, 200), 7, 0), ((200, 600), 12, 1), ((300, 300), 3, 2),
                                          ((256, 64), 0, 3), ((500, 100), 40, 4)])
def test_optimal_rank_matches_oracle(shape, k, seed):
    """Low-rank signal plus white noise: the product's rank equals the oracle's."""
    from dsmezo_b200.calibration import activation_rank, optimal_rank
    g = torch.Generator().manual_seed(seed)
    m, n = shape
    X = torch.randn(m, n, generator=g)
    if k:
        X += 4.0 * math.sqrt(max(m, n)) ** 0.5 * (torch.randn(m, k, generator=g) @ torch.randn(k, n, generator=g)) / k ** 0.5
    sv = torch.linalg.svdvals(X).numpy()
    beta = min(m, n) / max(m, n)
    assert optimal_rank(sv, beta) == ref.optht_rank(sv, beta)
    assert activation_rank(X) == ref.optht_rank(sv, beta)


def test_optimal_rank_edges():
    from dsmezo_b200.calibration import calibration_rank, optimal_rank
    assert optimal_rank(np.ones(10, dtype=np.float32), 0.5) == 0          # nothing above the cutoff
    sv = np.array([100.0, 1.0, 1.0, 1.0, 1.0], dtype=np.float32)
    assert optimal_rank(sv, 1.0) == 1
    with pytest.raises(ValueError):
        optimal_rank(sv, 1.5)
    # the median of the ranks, truncated (ds_mezo/controller.py:154)
    g = torch.Generator().manual_seed(3)
    acts = [torch.randn(120, 60, generator=g) for _ in range(2)]
    acts[0] += 30 * torch.randn(120, 1, generator=g) @ torch.randn(1, 60, generator=g)
    ranks = [ref.optht_rank(torch.linalg.svdvals(a).numpy(), 0.5) for a in acts]
    assert calibration_rank(acts) == int(np.median(ranks))


@pytest.mark.parametrize("T,D,q,niter", [(300, 80, 10, 3), (60, 200, 8, 3), (128, 128, 16, 2), (90, 70, 5, 0)])
def test_oracle_svd_lowrank_matches_torch(T, D, q, niter):
    """The oracle restatement (fp32 here) against torch.svd_lowrank with the same sketch:
    torch draws torch.randn(rows, q) as its first random op."""
    g = torch.Generator().manual_seed(T + D)
    H = torch.randn(T, D, generator=g) * torch.exp(torch.randn(D, generator=g))
    rows = D if T >= D else T
    torch.manual_seed(11)
    sketch = torch.randn(rows, q)
    torch.manual_seed(11)
    _, S_t, V_t = torch.svd_lowrank(H, q=q, niter=niter)
    V_o, S_o = ref.svd_lowrank_sketched(H, sketch, niter, dtype=torch.float32)
    assert torch.allclose(S_o, S_t, rtol=1e-4, atol=0)
    for j in range(q):
        d = min(float((V_o[:, j] - V_t[:, j]).norm()), float((V_o[:, j] + V_t[:, j]).norm()))
        assert d < 1e-3
    # fp64 restatement spans the same subspace
    V_64, _ = ref.svd_lowrank_sketched(H, sketch, niter)
    assert ref.subspace_sine(V_t, V_64) < 1e-4


def test_basis_draw_increments_follow_svd_lowrank_shapes():
    from dsmezo_b200 import transformer_adapter_shapes
    from dsmezo_b200.calibration import basis_draw_increments
    from dsmezo_b200._lib import lib
    _, bases = transformer_adapter_shapes(1, 512, 1408, 128, 1024)
    inc = basis_draw_increments(bases, 8, 148, 2048)
    L = lib()
    want = [int(L.dsmz_randn_offset_increment((b.D if b.T >= b.D else b.T) * 8, 148, 2048)) for b in bases]
    assert inc == want
    assert bases[3].T < bases[3].D and bases[0].T >= bases[0].D


def _rank_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from dsmezo_b200.calibration import calibration_rank
        g = torch.Generator().manual_seed(rank)
        acts = [torch.randn(100, 50, generator=g) + (10 + 5 * i) * torch.randn(100, 2 + i + rank, generator=g)
                @ torch.randn(2 + i + rank, 50, generator=g) for i in range(2)]
        results[rank] = calibration_rank(acts, process_group=dist.group.WORLD)
    finally:
        dist.destroy_process_group()


def test_calibration_rank_over_ranks():
    from dsmezo_b200.calibration import activation_rank
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    allr = []
    for rank in range(2):
        g = torch.Generator().manual_seed(rank)
        acts = [torch.randn(100, 50, generator=g) + (10 + 5 * i) * torch.randn(100, 2 + i + rank, generator=g)
                @ torch.randn(2 + i + rank, 50, generator=g) for i in range(2)]
        allr += [activation_rank(a) for a in acts]
    assert results[0] == results[1] == int(np.median(allr))
