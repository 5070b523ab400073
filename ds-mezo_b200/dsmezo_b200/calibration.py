"""First-step calibration of the activation bases (ds_mezo/controller.py:135-163).

The reference, on the first step:
  1. takes the singular values of every unique activation H (T x D) with
     torch.linalg.svdvals and picks a rank for each with optht (the optimal hard threshold
     of Gavish & Donoho, "The Optimal Hard Threshold for Singular Values is 4/sqrt(3)",
     IEEE Trans. Inf. Theory 60(8), 2014, noise level unknown); the basis width is the
     median of those ranks, truncated to an int (controller.py:137-154);
  2. sets every basis to V of torch.svd_lowrank(H, q=width, niter) (controller.py:156-163).

Step 1 is host arithmetic on the full spectrum; its singular values come from the same
library call the reference makes (torch.linalg.svdvals on the device, once per run). Step 2
is dsmz_plan_calibrate: one batched randomized SVD of all bases on the plan's power-iteration
kernels (AdapterSet.calibrate).
"""
from __future__ import annotations

import math
from typing import Iterable, Optional, Sequence

import numpy as np
import torch


def marchenko_pastur_cdf(x: float, beta: float) -> float:
    """CDF of the Marchenko-Pastur law with aspect ratio beta in (0, 1] and unit variance
    (support [(1 - sqrt(beta))^2, (1 + sqrt(beta))^2], density
    sqrt((b - x)(x - a)) / (2 pi beta x)). With x = c - h cos(t), c = 1 + beta,
    h = 2 sqrt(beta), the integral has the closed form
      F = (2/pi) [sin t / (2 sqrt beta) + (1 + beta) t / (4 beta)
                  - (1 - beta) / (2 beta) * atan((1 + sqrt beta) / (1 - sqrt beta) * tan(t / 2))]."""
    if not 0.0 < beta <= 1.0:
        raise ValueError("beta must be in (0, 1]")
    sb = math.sqrt(beta)
    a, b = (1.0 - sb) ** 2, (1.0 + sb) ** 2
    if x <= a:
        return 0.0
    if x >= b:
        return 1.0
    c, h = 1.0 + beta, 2.0 * sb
    t = math.acos(min(1.0, max(-1.0, (c - x) / h)))
    g = math.sin(t) / (2.0 * sb) + c * t / (4.0 * beta)
    if beta < 1.0:
        g -= (1.0 - beta) / (2.0 * beta) * math.atan((1.0 + sb) / (1.0 - sb) * math.tan(0.5 * t))
    return 2.0 / math.pi * g


def marchenko_pastur_median(beta: float) -> float:
    """Median of the Marchenko-Pastur law (bisection on the closed-form CDF to fp64
    resolution)."""
    sb = math.sqrt(beta)
    lo, hi = (1.0 - sb) ** 2, (1.0 + sb) ** 2
    for _ in range(200):
        mid = 0.5 * (lo + hi)
        if mid == lo or mid == hi:
            break
        if marchenko_pastur_cdf(mid, beta) < 0.5:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def optimal_threshold_known_noise(beta: float) -> float:
    """lambda*(beta) = sqrt(2 (beta + 1) + 8 beta / (beta + 1 + sqrt(beta^2 + 14 beta + 1)))
    (Gavish & Donoho, eq. 11): the threshold over sqrt(n) sigma for a known noise level."""
    return math.sqrt(2.0 * (beta + 1.0) + 8.0 * beta / (beta + 1.0 + math.sqrt(beta * beta + 14.0 * beta + 1.0)))


def optimal_threshold_coefficient(beta: float) -> float:
    """omega(beta) = lambda*(beta) / sqrt(mu_beta) with mu_beta the Marchenko-Pastur median:
    the threshold over the median singular value when the noise level is unknown."""
    return optimal_threshold_known_noise(beta) / math.sqrt(marchenko_pastur_median(beta))


def optimal_rank(sv, beta: float) -> int:
    """Number of singular values above omega(beta) * median(sv) (sv in descending order, as
    svdvals returns them, so the count is the reference's last index above the cutoff + 1)."""
    if not 0.0 < beta <= 1.0:
        raise ValueError("beta must be in (0, 1]")
    sv = np.asarray(sv)
    cutoff = optimal_threshold_coefficient(beta) * np.median(sv)
    above = np.nonzero(sv > cutoff)[0]
    return int(above.max()) + 1 if above.size else 0


def activation_rank(H: torch.Tensor) -> int:
    """optht rank of one activation (ds_mezo/controller.py:149-153): its singular values in
    fp32 on its device (the reference's hooks hand over fp32 activations)."""
    sv = torch.linalg.svdvals(H.float()).cpu().numpy()
    m, n = H.shape
    return optimal_rank(sv, min(m, n) / max(m, n))


def calibration_rank(activations: Iterable[torch.Tensor], process_group=None) -> int:
    """Basis width of the first step: the median of the unique activations' optht ranks,
    truncated to an int (ds_mezo/controller.py:154). With a process group, each rank passes
    its own activations and the median is taken over all of them."""
    ranks = [activation_rank(h) for h in activations]
    if process_group is not None:
        import torch.distributed as dist
        gathered = [None] * dist.get_world_size(process_group)
        dist.all_gather_object(gathered, ranks, group=process_group)
        ranks = [r for part in gathered for r in part]
    if not ranks:
        raise ValueError("no activations")
    return int(np.median(ranks))


def basis_draw_increments(bases: Sequence, width: int, sm_count: int, max_threads_per_sm: int) -> list:
    """Generator advance of each basis's svd_lowrank sketch: torch.randn(D, width) when
    T >= D, torch.randn(T, width) when T < D."""
    from ._lib import lib
    L = lib()
    return [int(L.dsmz_randn_offset_increment((b.D if b.T >= b.D else b.T) * width, sm_count, max_threads_per_sm))
            for b in bases]


def generator_of(device: torch.device, generator: Optional[torch.Generator]) -> torch.Generator:
    """The generator svd_lowrank would draw from: the device's default CUDA generator unless
    one is given."""
    if generator is not None:
        return generator
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return torch.cuda.default_generators[idx]
