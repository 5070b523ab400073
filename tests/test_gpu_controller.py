"""The controller's perturbation scale on the GPU: the Frobenius norms of the fp32 masters
(one grouped launch pair) and eps = median norm x FLT_EPSILON^(1/3) against the value the
reference's own DSMeZO_Controller computed for the recorded adapters (tests/golden/
controller_mini.pt, ds_mezo/controller.py:78-82)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_factor_norms_and_eps_match_the_reference_controller():
    from dsmezo_b200 import AdapterSet, ZOController, transformer_adapter_shapes
    mini = torch.load("tests/golden/controller_mini.pt", weights_only=False)
    cfg = mini["config"]
    mods, bases = transformer_adapter_shapes(cfg["layers"], cfg["h"], cfg["inter"], cfg["kv"], cfg["T"])
    aset = AdapterSet(mods, bases, cfg["r"], cfg["r"], copy_dtype=torch.float32, act_dtype=torch.float32, device=DEV)
    for i, m in enumerate(mods):
        st = mini["init"][f"{m.layer}.{m.name}"]
        aset.A(i).copy_(st["A"])
        aset.B(i).copy_(st["B"])
    norms = aset.factor_norms().cpu()
    want = torch.stack([torch.linalg.norm(mini["init"][f"{m.layer}.{m.name}"][k].double())
                        for m in mods for k in ("A", "B")])
    assert torch.allclose(norms.double(), want, rtol=1e-6, atol=0)
    gen = torch.Generator(device=DEV).manual_seed(0)
    ctl = ZOController.from_factors(aset, cfg["total_steps"], gen)
    assert math.isclose(ctl.eps, cfg["eps"], rel_tol=1e-6)
    assert math.isclose(ctl.eta_max, cfg["eta_max"], rel_tol=1e-6)
    assert math.isclose(ctl.eta_min, cfg["eta_min"], rel_tol=1e-6)


@pytest.mark.parametrize("shape", [(3584, 64), (64, 18944), (5, 3)])
def test_factor_norms_large_and_ragged(shape):
    from dsmezo_b200 import AdapterSet, ModuleShape, BasisShape
    d_out, d_in = (shape[0], 300) if shape[1] < shape[0] else (300, shape[1])
    r = min(shape)
    mods = [ModuleShape(0, "q_proj", d_out, d_in, 0)]
    bases = [BasisShape(0, "qkv", 16, d_in)]
    aset = AdapterSet(mods, bases, r, r, copy_dtype=torch.bfloat16, act_dtype=torch.bfloat16, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(1)
    aset.factors.normal_(generator=g)
    norms = aset.factor_norms().double().cpu()
    want = torch.tensor([float(torch.linalg.norm(aset.A(0).double())), float(torch.linalg.norm(aset.B(0).double()))],
                        dtype=torch.float64)
    assert torch.allclose(norms, want, rtol=1e-6, atol=0)
