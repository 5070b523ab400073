"""Pins the CPU oracle against golden vectors produced by the reference's own code.

The fixtures come from tests/golden/make_golden.py, which ran ds_mezo/kernels.py
(Triton interpreter) and ds_mezo/controller.py on CPU. CPU only.
"""
import math
from pathlib import Path

import pytest
import torch

from oracle import reference_ops as ref

GOLD = Path(__file__).resolve().parent / "golden"
FLOOR = ref.FLT_MIN


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


@pytest.fixture(scope="module")
def kern():
    return torch.load(GOLD / "kernels.pt", weights_only=False)


@pytest.fixture(scope="module")
def mini():
    return torch.load(GOLD / "controller_mini.pt", weights_only=False)


def test_cubic_schedule_matches_reference(kern):
    sched = ref.ns_cubic_schedule()
    assert len(sched) == 12
    c1 = torch.tensor([s[0] for s in sched], dtype=torch.float64)
    c3 = torch.tensor([s[1] for s in sched], dtype=torch.float64)
    assert torch.equal(c1, kern["ns_c1"]) and torch.equal(c3, kern["ns_c3"])


def test_power_iters_is_three():
    assert ref.svd_power_iters() == 3


@pytest.mark.parametrize("name", ["tall_1408x8", "tall_200x16", "tall_16x16", "wide_8x512", "wide_16x1000",
                                  "wide_4x37"])
def test_zo_muon(kern, name):
    c = kern[f"muon_{name}"]
    param = c["param_in"].clone()
    scratch = torch.zeros_like(param)
    ref.zo_muon_update(param, c["buf"], scratch, c["eta"], FLOOR)
    assert rel(scratch, c["scratch_out"]) < 2e-6
    assert rel(param - c["param_in"], c["param_out"] - c["param_in"]) < 2e-5


@pytest.mark.parametrize("name", ["t256_d512_r8", "t64_d200_r8", "t130_d96_r16", "t32_d48_r5"])
def test_power_iter(kern, name):
    c = kern[f"pi_{name}"]
    V = ref.fused_power_iter(c["H"], c["V0"], c["iters"], FLOOR)
    # same basis (not only the same span): MGS is deterministic up to fp32 rounding
    assert rel(V, c["V"]) < 1e-4
    assert ref.subspace_sine(V, c["V"]) < 1e-5


@pytest.mark.parametrize("name", ["q_128x8x512_rc8", "o_300x8x200_rc4", "k_64x4x96_rc8", "g_704x16x256_rc16"])
def test_agzo(kern, name):
    c = kern[f"agzo_{name}"]
    z_A, z_B = ref.fused_agzo_perturbation(c["B"], c["V"], c["zcB"], c["zcA"], c["eps"], FLOOR)
    assert rel(z_B, c["z_B"]) < 1e-6
    assert rel(z_A, c["z_A"]) < 1e-5


def test_dual(kern):
    c = kern["dual"]
    pos, neg = torch.empty(1000), torch.empty(1000)
    ref.fused_perturb_dual(c["base"], c["z"], pos, neg)
    assert torch.equal(pos, c["pos"]) and torch.equal(neg, c["neg"])


def _state_from_golden(mini):
    cfg = mini["config"]
    groups = {"qkv": ("q_proj", "k_proj", "v_proj"), "o": ("o_proj",), "gu": ("gate_proj", "up_proj"),
              "down": ("down_proj",)}
    mod2g = {m: g for g, ms in groups.items() for m in ms}
    gnames = list(groups)
    bases = []
    for li in range(cfg["layers"]):
        for gname in gnames:
            bases.append(mini["bases0"][f"{li}.{gname}"].clone())
    mods = []
    for li in range(cfg["layers"]):
        for name in ref.MODULE_ORDER:
            s = mini["init"][f"{li}.{name}"]
            mods.append(ref.Module(li, name, s["A"].clone(), s["B"].clone(), s["mu_A"].clone(), s["mu_B"].clone(),
                                   s["var_A"].clone(), s["var_B"].clone(), basis=li * 4 + gnames.index(mod2g[name])))
    st = ref.StepState(mods, bases, eps=cfg["eps"], total_steps=cfg["total_steps"])
    assert math.isclose(st.eta_max, cfg["eta_max"]) and math.isclose(st.eta_min, cfg["eta_min"])
    return st, gnames


def test_controller_steps_match_reference(mini):
    """Two full optimizer steps of the reference controller (power iteration, AGZO,
    dual perturb, Kalman, ZO-Muon, cosine eta) reproduced by the oracle."""
    st, gnames = _state_from_golden(mini)
    A0 = [m.A for m in st.modules]
    B0 = [m.B for m in st.modules]
    assert math.isclose(ref.eps_from_factors(A0, B0), mini["config"]["eps"], rel_tol=1e-6)
    cfg = mini["config"]
    for step in mini["steps"]:
        acts = [step["activations"][f"{li}.{g}"] for li in range(cfg["layers"]) for g in gnames]
        st.step_count += 1
        assert st.step_count == step["step_count"]
        assert math.isclose(st.eta, step["eta"], rel_tol=1e-12)
        shapes = ref.draw_shapes(st.modules, st.bases)
        assert [tuple(d.shape) for d in step["draws"]] == shapes
        perts = ref.perturb_phase(st, acts, step["draws"], cfg["power_iter_steps"])
        for i, li in enumerate(range(cfg["layers"])):
            for gname in gnames:
                assert rel(st.bases[li * 4 + gnames.index(gname)], step["bases"][f"{li}.{gname}"]) < 1e-4
        for m, (z_A, z_B) in zip(st.modules, perts):
            key = f"{m.layer}.{m.name}"
            gzA, gzB = step["z"][key]
            assert rel(z_A, gzA) < 1e-4 and rel(z_B, gzB) < 1e-4
            assert rel(m.pos_A - m.A, step["pos"][key][0] - m.A) < 1e-4
        ref.update_phase(st, perts, step["dd"])
        assert math.isclose(st.eta, step["eta_after"], rel_tol=1e-12)
        for m in st.modules:
            g = step["state"][f"{m.layer}.{m.name}"]
            for k in ("mu_A", "mu_B", "var_A", "var_B"):
                assert rel(getattr(m, k), g[k]) < 1e-4, k
            a0 = mini["init"][f"{m.layer}.{m.name}"]
            assert rel(m.A - a0["A"], g["A"] - a0["A"]) < 1e-3
            assert rel(m.B - a0["B"], g["B"] - a0["B"]) < 1e-3


def test_contrastive_loss_matches_reference():
    # the reference's _score_contrastive on a stub backend (tests/golden/make_golden.py)
    cases = torch.load(GOLD / "scoring.pt", weights_only=False)
    assert len(cases) == 4
    for c in cases:
        for k in ("pos", "neg"):
            got = ref.contrastive_loss(c[f"rows_{k}"], c["targets"].tolist(), c["seq_tokens"], c["advantages"])
            assert got == c[f"loss_{k}"], (k, got, c[f"loss_{k}"])
