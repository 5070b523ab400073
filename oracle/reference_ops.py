"""ORACLE: CPU restatement of DS-MeZO's zeroth-order optimizer hot path.

This module is test infrastructure. Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference`` arm) may import it,
and only as the checker or as the timed CPU baseline. The product package
(``dsmezo_b200``) never imports it and has no CPU fallback.

Every function is plain fp32 torch-on-CPU arithmetic that follows the reference op by
op. Citations are ``path:line`` inside the reference project:

* ``ds_mezo/kernels.py:5-24``     Newton-Schulz cubic schedule      -> ``ns_cubic_schedule``
* ``ds_mezo/kernels.py:26-186``   ZO-Muon tall/wide NS + update     -> ``zo_muon_update``
* ``ds_mezo/kernels.py:188-265``  activation power iteration + MGS  -> ``fused_power_iter``
* ``ds_mezo/kernels.py:267-397``  AGZO perturbation                 -> ``fused_agzo_perturbation``
* ``ds_mezo/kernels.py:399-422``  dual perturb                      -> ``fused_perturb_dual``
* ``ds_mezo/controller.py:14-15, 194-201``  contrastive scoring loss -> ``contrastive_loss``
* ``ds_mezo/controller.py:78-88, 178-193, 216-229, 236-292``        -> controller helpers below

The restatement is pinned against golden vectors that the reference's own Triton kernels
and controller produced (run under ``TRITON_INTERPRET=1`` on CPU); the generator script
is ``tests/golden/make_golden.py`` and the check is ``tests/test_oracle_golden.py``.
The torch CUDA Philox stream that the reference controller draws from cannot run on a
CPU; CPU checks inject the recorded Gaussian draws instead, and the bit-exact stream
check runs on the GPU against ``torch.randn(generator=cuda_generator)``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

FLT_MIN = float(torch.finfo(torch.float32).tiny)   # norm_floor, ds_mezo/controller.py:108
FLT_EPS = float(torch.finfo(torch.float32).eps)

MODULE_ORDER = ("down_proj", "gate_proj", "k_proj", "o_proj", "q_proj", "up_proj", "v_proj")
"""Per-layer module order: ``discover_layers`` sorts specs by (layer_idx, module_name)
(ds_mezo/model_config.py:37), which fixes the order of the random draws."""


# --------------------------------------------------------------------------------------
# Newton-Schulz schedules
# --------------------------------------------------------------------------------------
def ns_cubic_schedule() -> Tuple[Tuple[float, float, float], ...]:
    """Degree-3 minimax schedule of ds_mezo/kernels.py:5-24.

    Returns (a0, a1, a2) triples for S = a0*I + a1*G + a2*G^2 (a2 = 0 here), so that one
    iteration is X <- X S (tall) or X <- S X (wide). The recurrence on the interval
    [l, u] runs until 1 - l < eps_f32, which gives 12 steps.
    """
    eps = FLT_EPS
    lo, up = eps ** 0.5, 1.0
    out = []
    while 1.0 - lo >= eps:
        s = up * up + lo * up + lo * lo
        alpha = (3.0 / s) ** 0.5
        alpha3 = alpha * alpha * alpha
        beta = 4.0 / (2.0 + lo * up * (lo + up) * alpha3)
        c1 = 1.5 * beta * alpha
        c3 = -0.5 * beta * alpha3
        out.append((c1, c3, 0.0))
        lo = c1 * lo + c3 * lo * lo * lo
        up = 2.0 - lo
    return tuple(out)


QUINTIC_MUON_SCHEDULE = tuple((3.4445, -4.7750, 2.0315) for _ in range(5))
"""Five quintic Muon steps X <- aX + b(XX^T)X + c(XX^T)^2 X, the schedule the toy and
1.5B-shaped benchmark sets name. Not in the reference kernels; written in the same
S = a0 I + a1 G + a2 G^2 form."""


def get_schedule(name: str):
    if name == "cubic":
        return ns_cubic_schedule()
    if name == "quintic":
        return QUINTIC_MUON_SCHEDULE
    raise ValueError(f"unknown Newton-Schulz schedule {name!r}")


# --------------------------------------------------------------------------------------
# ds_mezo/kernels.py restatements
# --------------------------------------------------------------------------------------
def _poly(G: torch.Tensor, coeffs) -> torch.Tensor:
    a0, a1, a2 = coeffs
    eye = torch.eye(G.shape[0], dtype=G.dtype)
    S = a0 * eye + a1 * G
    if a2 != 0.0:
        S = S + a2 * (G @ G)
    return S


def ns_orthogonalize(buf: torch.Tensor, norm_floor: float = FLT_MIN, schedule=None,
                     dtype=torch.float32) -> torch.Tensor:
    """X_final of ds_mezo/kernels.py:26-164: Frobenius-normalise, then iterate in X space.

    Tall (M >= N, ds_mezo/kernels.py:169) uses G = X^T X and X <- X S; wide uses
    G = X X^T and X <- S X. fp32 without TF32 by default, like ``allow_tf32=False``;
    ``dtype=torch.float64`` gives the same algorithm without its fp32 rounding.
    """
    sched = ns_cubic_schedule() if schedule is None else schedule
    X = buf.detach().to(dtype).clone()
    M, N = X.shape
    norm_sq = (X * X).sum()
    inv_norm = 1.0 / torch.sqrt(torch.clamp(norm_sq, min=norm_floor))
    X = X * inv_norm
    tall = M >= N
    for coeffs in sched:
        G = X.T @ X if tall else X @ X.T
        S = _poly(G, coeffs)
        X = X @ S if tall else S @ X
    return X


def zo_muon_update(param, buf, scratch, eta, norm_floor=FLT_MIN, schedule=None):
    """ds_mezo/kernels.py:167-186: scratch <- NS(buf); param <- param - eta * scratch.

    Arithmetic runs in buf's dtype (fp32 in the reference; fp64 for the exact variant).
    """
    cdt = torch.float64 if buf.dtype == torch.float64 else torch.float32
    X = ns_orthogonalize(buf, norm_floor, schedule, cdt)
    scratch.copy_(X)
    step = X * torch.tensor(eta, dtype=cdt)   # eta * orth in the compute dtype, as the kernel does
    if param.dtype == cdt:
        param.sub_(step)
    else:  # bf16 factors: compute-dtype arithmetic, one rounding on store
        param.copy_((param.to(cdt) - step).to(param.dtype))


def mgs_columns(W: torch.Tensor, norm_floor: float, ncols: Optional[int] = None,
                dtype=torch.float32) -> torch.Tensor:
    """Modified Gram-Schmidt over the first ``ncols`` columns, in place semantics of
    ds_mezo/kernels.py:227-240 (power iteration) and :328-340 (AGZO).

    Each column is orthogonalised against the already-normalised earlier columns with the
    running vector (MGS, not CGS), then divided by sqrt(max(|v|^2, norm_floor)).
    Columns past ``ncols`` are left as they are.
    """
    Q = W.detach().to(dtype).clone()
    n = Q.shape[1] if ncols is None else ncols
    for col in range(n):
        v = Q[:, col].clone()
        for prev in range(col):
            q = Q[:, prev]
            v = v - torch.dot(v, q) * q
        nrm = torch.sqrt(torch.clamp(torch.dot(v, v), min=norm_floor))
        Q[:, col] = v / nrm
    return Q


def fused_power_iter(H, V, num_iters, norm_floor=FLT_MIN, dtype=torch.float32):
    """ds_mezo/kernels.py:188-265: num_iters x {W = H^T (H V); V = MGS(W)}; returns D x R."""
    Hf = H.detach().to(dtype)
    Vk = V.detach().to(dtype).clone()
    for _ in range(num_iters):
        W = Hf.T @ (Hf @ Vk)
        Vk = mgs_columns(W, norm_floor, dtype=dtype)
    return Vk.contiguous()


def fused_agzo_perturbation(B, V, z_coeff_B, z_coeff_A, eps, norm_floor=FLT_MIN, dtype=torch.float32):
    """ds_mezo/kernels.py:267-397.

    z_B = eps * Zc_B V^T (R x d_in); BV = B V (R x RC); Q = MGS over the first
    RC_A = min(R, RC) columns of BV; z_A = eps * Zc_A Q[:, :RC_A]^T (d_out x R).
    """
    assert z_coeff_B.is_contiguous() and z_coeff_A.is_contiguous()
    Bf = B.detach().to(dtype)
    Vf = V.detach().to(dtype)
    R, _ = Bf.shape
    RC = Vf.shape[1]
    rca = min(R, RC)
    z_B = (z_coeff_B.to(dtype) @ Vf.T) * eps
    BV = Bf @ Vf
    Q = mgs_columns(BV, norm_floor, rca, dtype)
    z_A = (z_coeff_A.to(dtype) @ Q[:, :rca].T) * eps
    return z_A.contiguous(), z_B.contiguous()


def fused_perturb_dual(base, z, pos, neg):
    """ds_mezo/kernels.py:399-422: pos = base + z, neg = base - z (flat, contiguous)."""
    cdt = torch.float64 if (base.dtype == torch.float64 or z.dtype == torch.float64) else torch.float32
    b = base.reshape(-1).to(cdt)
    zz = z.reshape(-1).to(cdt)
    pos.view(-1).copy_((b + zz).to(pos.dtype))
    neg.view(-1).copy_((b - zz).to(neg.dtype))


def subspace_sine(V: torch.Tensor, V_ref: torch.Tensor) -> float:
    """Largest principal-angle sine between span(V) and span(V_ref).

    Both are orthonormalised in fp64 first; the sine is the spectral norm of the part of
    V_ref outside span(V), which stays accurate for tiny angles (1 - cos^2 does not).
    """
    Q = torch.linalg.qr(V.detach().double())[0]
    Qr = torch.linalg.qr(V_ref.detach().double())[0]
    resid = Qr - Q @ (Q.T @ Qr)
    return float(torch.linalg.matrix_norm(resid, ord=2))


# --------------------------------------------------------------------------------------
# ds_mezo/controller.py restatements
# --------------------------------------------------------------------------------------
def svd_power_iters() -> int:
    """ds_mezo/model_config.py:45-47 for fp32: ceil(log3(log2(1/eps))) = 3."""
    return math.ceil(math.log(math.log(1.0 / FLT_EPS) / math.log(2.0)) / math.log(3.0))


def eps_from_factors(A_list: Sequence[torch.Tensor], B_list: Sequence[torch.Tensor]) -> float:
    """ds_mezo/controller.py:78-82: median Frobenius norm of all factors times eps^(1/3)."""
    norms = torch.stack([torch.linalg.norm(a.float()) for a in A_list]
                        + [torch.linalg.norm(b.float()) for b in B_list])
    return float(torch.median(norms)) * FLT_EPS ** (1.0 / 3.0)


def eta_bounds(eps: float) -> Tuple[float, float]:
    """ds_mezo/controller.py:84-88: (eta_max, eta_min) = (eps, eps * eps_f32^(1/3))."""
    return eps, eps * FLT_EPS ** (1.0 / 3.0)


def cosine_eta(step: int, total_steps: int, eta_max: float, eta_min: float) -> float:
    """ds_mezo/controller.py:290-292."""
    return eta_min + 0.5 * (eta_max - eta_min) * (1.0 + math.cos(math.pi * step / total_steps))


def kalman_beta_q(step_count: int, total_steps: int, eps: float) -> Tuple[float, float]:
    """ds_mezo/controller.py:255-258: beta = 1 - 1/min(step, floor(sqrt(T))); q = eps^2 (1 - beta^2)."""
    max_window = int(math.sqrt(total_steps))
    beta = 1.0 - 1.0 / min(step_count, max_window)
    q = eps ** 2 * (1.0 - beta * beta)
    return beta, q


def get_perturbation(A, B, V, var_B, randn_B, randn_A, eps, norm_floor=FLT_MIN, dtype=torch.float32):
    """ds_mezo/controller.py:178-193 with the two Gaussian draws injected.

    randn_B: R x RC standard normals (first draw), randn_A: d_out x min(R, RC) (second draw).
    """
    var_B_proj = var_B.to(dtype) @ (V.to(dtype) ** 2)
    z_coeff_B = randn_B.to(dtype) * torch.sqrt(var_B_proj)
    z_coeff_A = randn_A.to(dtype).contiguous()
    return fused_agzo_perturbation(B, V, z_coeff_B.contiguous(), z_coeff_A, eps, norm_floor, dtype)


def shrinkage_rloo(rewards: Sequence[float], reward_ema: float, momentum: float,
                   norm_floor: float = FLT_MIN):
    """ds_mezo/controller.py:216-229: James-Stein shrinkage of the RLOO baseline.

    Returns (advantages, new_reward_ema).
    """
    r = torch.tensor(list(rewards))
    n = len(rewards)
    r_bar = float(r.mean())
    base_rloo = (r.sum() - r) / (n - 1)
    rvar = float(r.var())
    lam = rvar / (rvar + (r_bar - reward_ema) ** 2 + norm_floor)
    base = (1.0 - lam) * base_rloo + lam * reward_ema
    adv = (r - base).tolist()
    new_ema = momentum * reward_ema + (1.0 - momentum) * r_bar
    return adv, new_ema


def contrastive_loss(rows: torch.Tensor, targets: Sequence[int], seq_tokens: Sequence[int],
                     advantages: Sequence[float]) -> float:
    """ds_mezo/controller.py:194-201 with _mean_nll (:14-15): sum_i adv_i * mean NLL of
    sequence i's scored tokens. rows holds the logits that predict each scored token (one
    row per token, sequences one after another); the logprob of a token is the fp32
    log-softmax entry vLLM reports (ds_mezo/backend.py:98-103), turned into a Python float,
    and the sums run over Python floats in the reference's order."""
    lp = torch.log_softmax(rows.float(), dim=-1)
    vals = [float(lp[j, int(t)]) for j, t in enumerate(targets)]
    loss, o = 0, 0
    for adv, n in zip(advantages, seq_tokens):
        seq = vals[o:o + n]
        loss = loss + adv * (-sum(seq) / len(seq))
        o += n
    return float(loss)


def rloo_advantages(rewards: Sequence[float]) -> List[float]:
    """Plain RLOO baseline (sum - r)/(N - 1) (README.md:18-21), used by the many-direction set."""
    r = torch.tensor(list(rewards), dtype=torch.float64)
    n = len(rewards)
    return (r - (r.sum() - r) / (n - 1)).tolist()


@dataclass
class Matrix:
    """One factor of one adapter with its Kalman state (ds_mezo/controller.py:18-34)."""
    param: torch.Tensor
    mu: torch.Tensor
    var: torch.Tensor
    scratch: torch.Tensor


def kalman_update(mats: Sequence[Matrix], zs: Sequence[torch.Tensor], dd: float, beta: float, q: float,
                  eta: float, norm_floor: float = FLT_MIN, schedule=None, scratch_out: bool = True):
    """ds_mezo/controller.py:260-286, in the reference's op order and fp32 rounding.

    ``mats`` and ``zs`` run in the controller's order: for each module (layer, name), A then B.
    Returns (y_hat, s_sum) as fp32 0-d tensors for inspection.
    """
    cdt = mats[0].mu.dtype if mats else torch.float32
    y_hat = torch.zeros((), dtype=cdt)
    s_sum = torch.zeros((), dtype=cdt)
    for m, z in zip(mats, zs):
        m.mu.mul_(beta)
        m.var.mul_(beta * beta).add_(q)
        y_hat += (z * m.mu).sum()
        s_sum += (z * z * m.var).sum()
    S = s_sum + norm_floor
    innovation = dd - y_hat
    inv_S = 1.0 / S
    for m, z in zip(mats, zs):
        K = m.var * z * inv_S
        m.mu.add_(innovation * K)
        m.var.mul_(1.0 - K * z)
        zo_muon_update(m.param, m.mu, m.scratch, eta, norm_floor, schedule)
    return y_hat, s_sum


# --------------------------------------------------------------------------------------
# Whole optimizer step over an adapter set (controller._perturb_and_sync + _update_weights)
# --------------------------------------------------------------------------------------
@dataclass
class Module:
    layer: int
    name: str
    A: torch.Tensor          # d_out x r
    B: torch.Tensor          # r x d_in
    mu_A: torch.Tensor
    mu_B: torch.Tensor
    var_A: torch.Tensor
    var_B: torch.Tensor
    basis: int               # index into the unique-activation list
    scratch_A: Optional[torch.Tensor] = None
    scratch_B: Optional[torch.Tensor] = None
    pos_A: Optional[torch.Tensor] = None
    pos_B: Optional[torch.Tensor] = None
    neg_A: Optional[torch.Tensor] = None
    neg_B: Optional[torch.Tensor] = None

    def __post_init__(self):
        for k in ("A", "B"):
            p = getattr(self, k)
            for pre in ("scratch_", "pos_", "neg_"):
                if getattr(self, pre + k) is None:
                    setattr(self, pre + k, torch.zeros_like(p, dtype=self.mu_A.dtype if pre == "scratch_" else p.dtype))


@dataclass
class StepState:
    modules: List[Module]
    bases: List[torch.Tensor]                    # one D x R basis per unique activation
    eps: float
    total_steps: int
    step_count: int = 0
    eta_max: float = 0.0
    eta_min: float = 0.0
    eta: float = 0.0
    schedule: tuple = field(default_factory=ns_cubic_schedule)
    dtype: torch.dtype = torch.float32     # float64: the same algorithm without fp32 rounding

    def __post_init__(self):
        if self.eta_max == 0.0:
            self.eta_max, self.eta_min = eta_bounds(self.eps)
            self.eta = self.eta_max


def draw_shapes(modules: Sequence[Module], bases: Sequence[torch.Tensor]):
    """The (rows, cols) of every Gaussian draw of one step, in controller order
    (ds_mezo/controller.py:184-191): per module Zc_B (R x RC) then Zc_A (d_out x min(R, RC))."""
    out = []
    for m in modules:
        R = m.B.shape[0]
        RC = bases[m.basis].shape[1]
        out.append((R, RC))
        out.append((m.A.shape[0], min(R, RC)))
    return out


def perturb_phase(st: StepState, activations: Sequence[torch.Tensor], draws: Sequence[torch.Tensor],
                  num_iters: int = 3, norm_floor: float = FLT_MIN):
    """ds_mezo/controller.py:236-251 (with :165-193): power iteration per unique
    activation, AGZO perturbation per module, then pos/neg = base +/- z.

    ``draws`` holds the Gaussian draws in ``draw_shapes`` order. Returns [(z_A, z_B)].
    """
    st.bases = [fused_power_iter(H, V, num_iters, norm_floor, st.dtype) for H, V in zip(activations, st.bases)]
    perts = []
    for i, m in enumerate(st.modules):
        V = st.bases[m.basis]
        z_A, z_B = get_perturbation(m.A, m.B, V, m.var_B, draws[2 * i], draws[2 * i + 1],
                                    st.eps, norm_floor, st.dtype)
        perts.append((z_A, z_B))
    for m, (z_A, z_B) in zip(st.modules, perts):
        fused_perturb_dual(m.A, z_A, m.pos_A, m.neg_A)
        fused_perturb_dual(m.B, z_B, m.pos_B, m.neg_B)
    return perts


def update_phase(st: StepState, perts, dd: float, norm_floor: float = FLT_MIN):
    """ds_mezo/controller.py:253-292 for the step ``st.step_count`` (already incremented)."""
    beta, q = kalman_beta_q(st.step_count, st.total_steps, st.eps)
    mats, zs = [], []
    for m, (z_A, z_B) in zip(st.modules, perts):
        mats.append(Matrix(m.A, m.mu_A, m.var_A, m.scratch_A))
        zs.append(z_A)
        mats.append(Matrix(m.B, m.mu_B, m.var_B, m.scratch_B))
        zs.append(z_B)
    y_hat, s_sum = kalman_update(mats, zs, dd, beta, q, st.eta, norm_floor, st.schedule)
    st.eta = cosine_eta(st.step_count, st.total_steps, st.eta_max, st.eta_min)
    return y_hat, s_sum


# --------------------------------------------------------------------------------------
# Many-direction SPSA (no reference counterpart: the reference perturbs and observes one
# direction per step). Direction k takes the draws that the k-th of K successive
# one-direction steps would take; the K observations update the Kalman state jointly
# with the diagonal of the innovation covariance.
# --------------------------------------------------------------------------------------
def perturb_phase_directions(st: StepState, activations: Sequence[torch.Tensor], draws_per_dir,
                             num_iters: int = 3, norm_floor: float = FLT_MIN):
    """Power iteration once, then the AGZO perturbation of every module for each direction
    (``draws_per_dir[k]`` in ``draw_shapes`` order). Returns [[(z_A, z_B)] per direction]."""
    st.bases = [fused_power_iter(H, V, num_iters, norm_floor, st.dtype) for H, V in zip(activations, st.bases)]
    out = []
    for draws in draws_per_dir:
        perts = []
        for i, m in enumerate(st.modules):
            V = st.bases[m.basis]
            perts.append(get_perturbation(m.A, m.B, V, m.var_B, draws[2 * i], draws[2 * i + 1],
                                          st.eps, norm_floor, st.dtype))
        out.append(perts)
    return out


def kalman_update_directions(mats: Sequence[Matrix], zs_per_dir, dds: Sequence[float], beta: float, q: float,
                             eta: float, norm_floor: float = FLT_MIN, schedule=None):
    """Joint observation of K directions: with mu1 = beta mu, var1 = beta^2 var + q,
    y_k = sum z_k mu1, s_k = sum z_k^2 var1, innov_k = dd_k - y_k, inv_k = 1 / (s_k + floor):
    mu2 = mu1 + var1 sum_k z_k inv_k innov_k, var2 = var1 (1 - var1 sum_k z_k^2 inv_k);
    then the ZO-Muon update of every factor. Returns [(y_k, s_k)]."""
    cdt = mats[0].mu.dtype if mats else torch.float32
    K = len(dds)
    for m in mats:
        m.mu.mul_(beta)
        m.var.mul_(beta * beta).add_(q)
    sums = []
    for k in range(K):
        y = torch.zeros((), dtype=cdt)
        s = torch.zeros((), dtype=cdt)
        for m, z in zip(mats, zs_per_dir[k]):
            y += (z * m.mu).sum()
            s += (z * z * m.var).sum()
        sums.append((y, s))
    innov = [dds[k] - sums[k][0] for k in range(K)]
    inv = [1.0 / (sums[k][1] + norm_floor) for k in range(K)]
    for j, m in enumerate(mats):
        am = torch.zeros_like(m.mu)
        av = torch.zeros_like(m.mu)
        for k in range(K):
            z = zs_per_dir[k][j]
            zi = z * inv[k]
            am += zi * innov[k]
            av += zi * z
        m.mu.add_(m.var * am)
        m.var.mul_(1.0 - m.var * av)
        zo_muon_update(m.param, m.mu, m.scratch, eta, norm_floor, schedule)
    return sums


def update_phase_directions(st: StepState, perts_per_dir, dds: Sequence[float], norm_floor: float = FLT_MIN):
    beta, q = kalman_beta_q(st.step_count, st.total_steps, st.eps)
    mats, zs = [], [[] for _ in perts_per_dir]
    for i, m in enumerate(st.modules):
        mats.append(Matrix(m.A, m.mu_A, m.var_A, m.scratch_A))
        mats.append(Matrix(m.B, m.mu_B, m.var_B, m.scratch_B))
        for k, perts in enumerate(perts_per_dir):
            zs[k].append(perts[i][0])
            zs[k].append(perts[i][1])
    sums = kalman_update_directions(mats, zs, dds, beta, q, st.eta, norm_floor, st.schedule)
    st.eta = cosine_eta(st.step_count, st.total_steps, st.eta_max, st.eta_min)
    return sums


def rloo_direction_scalars(rewards: torch.Tensor, eps: float) -> List[float]:
    """K directions' projected-gradient scalars: rewards (K, N), the first N/2 rollouts under
    the + copy; advantage = r - (sum - r) / (N - 1) within a direction; L = -mean advantage
    of a copy; dd = (L+ - L-) / (2 eps) (ds_mezo/controller.py:307 for the last step)."""
    K, N = rewards.shape
    out = []
    for k in range(K):
        r = [float(x) for x in rewards[k]]
        tot = sum(r)
        adv = [ri - (tot - ri) / (N - 1) for ri in r]
        lp = -sum(adv[: N // 2]) / (N // 2)
        lm = -sum(adv[N // 2:]) / (N // 2)
        out.append((lp - lm) / (2.0 * eps))
    return out


# --------------------------------------------------------------------------------------
# First-step calibration (ds_mezo/controller.py:135-163)
# --------------------------------------------------------------------------------------
def svd_lowrank_sketched(H: torch.Tensor, sketch: torch.Tensor, niter: int, dtype=torch.float64):
    """(V, S) of torch.svd_lowrank(H, q, niter) with its Gaussian sketch given instead of
    drawn. The algorithm is torch's (the reference pins torch 2.10.0, uv.lock:4003-4004):
    torch/_lowrank.py _svd_lowrank and get_approximate_basis, i.e. Halko, Martinsson & Tropp
    2009, Algorithms 4.4 and 5.1. It transposes H when T < D, so the sketch is (D, q) when
    T >= D and (T, q) when T < D (torch.randn(A.shape[-1], q) of the transposed A)."""
    A = H.to(dtype)
    T, D = A.shape
    tall = T >= D
    if not tall:
        A = A.T
    Q = torch.linalg.qr(A @ sketch.to(dtype)).Q
    for _ in range(niter):
        Q = torch.linalg.qr(A.T @ Q).Q
        Q = torch.linalg.qr(A @ Q).Q
    U, S, Vh = torch.linalg.svd(Q.T @ A, full_matrices=False)
    V, U = Vh.T, Q @ U
    if not tall:
        U, V = V, U
    return V, S


def calibrate_bases(activations: Sequence[torch.Tensor], sketches: Sequence[torch.Tensor], niter: int,
                    dtype=torch.float64):
    """ds_mezo/controller.py:156-163 over the unique activations in order, with the sketches
    of their svd_lowrank calls given: the calibrated bases and their Ritz singular values."""
    return [svd_lowrank_sketched(h, s, niter, dtype) for h, s in zip(activations, sketches)]


def mp_median_quadrature(beta: float) -> float:
    """Median of the Marchenko-Pastur law by numerical quadrature of its density
    sqrt((b - x)(x - a)) / (2 pi beta x) and root finding (scipy), an independent check of
    the product's closed-form CDF."""
    from scipy import integrate, optimize
    sb = math.sqrt(beta)
    a, b = (1 - sb) ** 2, (1 + sb) ** 2
    dens = lambda x: math.sqrt(max((b - x) * (x - a), 0.0)) / (2 * math.pi * beta * x)
    cdf = lambda x: integrate.quad(dens, a, x, epsabs=1e-14, epsrel=1e-13, limit=200)[0]
    return optimize.brentq(lambda x: cdf(x) - 0.5, a, b, xtol=1e-15, rtol=1e-15)


def optht_rank(sv, beta: float) -> int:
    """optht(beta, sv, sigma=None) (optht 0.2.0, uv.lock:2464-2465; used at
    ds_mezo/controller.py:153), from its paper (Gavish & Donoho 2014): the cutoff
    omega(beta) * median(sv), omega = lambda*(beta) / sqrt(MP median), and the rank is the
    last index above the cutoff plus one (0 when none is)."""
    import numpy as np
    lam = math.sqrt(2 * (beta + 1) + 8 * beta / (beta + 1 + math.sqrt(beta ** 2 + 14 * beta + 1)))
    omega = lam / math.sqrt(mp_median_quadrature(beta))
    sv = np.asarray(sv)
    idx = np.where(sv > omega * np.median(sv))[0]
    return int(np.max(idx)) + 1 if idx.size else 0
