"""On-device first-step calibration (ds_mezo/controller.py:156-163) against the oracle's
restatement of torch.svd_lowrank with the same sketches, and against torch.svd_lowrank
itself on the GPU (the call the reference makes).

Gates: the principal-angle sine between our basis and the oracle's (fp64, same sketch)
<= 1e-4 and against torch's fp32 GPU svd_lowrank <= 1e-3; each column equal to the oracle's
up to sign where its singular value is separated from its neighbours (relative gap >= 5%);
the Ritz singular values to 1e-4 relative; the generator advanced exactly as the
reference's svd_lowrank draws advance it."""
import pytest
import torch

from oracle import reference_ops as ref
from step_harness import make_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
SINE_ORACLE = 1e-4
SINE_TORCH = 1e-3
SV_REL = 1e-4
COL_TOL = 1e-3
GAP = 0.05


def _sketches(bases, R, gen):
    """The sketches svd_lowrank draws, in basis order, from a copy of the generator."""
    out = []
    for b in bases:
        rows = b.D if b.T >= b.D else b.T
        out.append(torch.randn(rows, R, device=DEV, generator=gen).cpu())
    return out


def _check_columns(V, Vo, S, what):
    R = S.numel()
    s = S.double()
    for j in range(R):
        nb = [abs(s[j] - s[k]) / s[j] for k in (j - 1, j + 1) if 0 <= k < R]
        if not nb or min(nb) < GAP:
            continue
        v, vo = V[:, j].double(), Vo[:, j].double()
        d = min(float((v - vo).norm()), float((v + vo).norm()))
        assert d <= COL_TOL, f"{what} column {j}: |v -/+ v_ref| {d:.2e}"


def _run(layers, hidden, inter, kv, R, tokens, act_dtype, flags_simt=False, niter=3, seed=5):
    from dsmezo_b200 import AdapterSet
    mods, bases, A, B, V0, H = make_inputs(layers, hidden, inter, kv, R, tokens, seed, torch.float32, act_dtype)
    aset = AdapterSet(mods, bases, R, R, copy_dtype=torch.float32, act_dtype=act_dtype, device=DEV,
                      tensor_core_power_iter=not flags_simt)
    for b in range(len(bases)):
        aset.H(b).copy_(H[b])
    gen = torch.Generator(device=DEV)
    gen.manual_seed(1234 + seed)
    gen.set_offset(8)
    twin = torch.Generator(device=DEV)
    twin.manual_seed(1234 + seed)
    twin.set_offset(8)
    sketches = _sketches(bases, R, twin)
    sv = aset.calibrate(generator=gen, niter=niter, singular_values=True)
    torch.cuda.synchronize()
    assert aset.device_error() == 0
    assert gen.get_offset() == twin.get_offset()
    oracle = ref.calibrate_bases([h.float() for h in H], sketches, niter)
    for b, (Vo, So) in enumerate(oracle):
        V = aset.V(b).cpu()
        what = f"basis {b} (T {bases[b].T}, D {bases[b].D})"
        assert torch.isfinite(V).all(), what
        sine = ref.subspace_sine(V, Vo)
        assert sine <= SINE_ORACLE, f"{what}: sine {sine:.2e}"
        ortho = float((V.double().T @ V.double() - torch.eye(R, dtype=torch.float64)).abs().max())
        assert ortho <= 1e-5, f"{what}: |V^T V - I| {ortho:.2e}"
        rel = float(((sv[b].cpu().double() - So) / So).abs().max())
        assert rel <= SV_REL, f"{what}: singular values rel {rel:.2e}"
        _check_columns(V, Vo, So, what)
    return aset, bases, H


@pytest.mark.parametrize("R,act_dtype", [(16, torch.bfloat16), (64, torch.bfloat16), (8, torch.float32)])
def test_calibration_matches_oracle(R, act_dtype):
    # qkv / o / gate_up inputs have T >= D, the down input T < D: both svd_lowrank branches
    _run(1, 384, 1280, 64, R, 768, act_dtype)


def test_calibration_cuda_core_path():
    _run(1, 256, 704, 64, 16, 512, torch.bfloat16, flags_simt=True)


def test_calibration_rank128():
    # R = 128: the Jacobi rotation lives in global memory, the Gram of Y at 8 x 8 per thread
    _run(1, 256, 640, 128, 128, 512, torch.bfloat16, niter=2)


@pytest.mark.parametrize("niter", [0, 1])
def test_calibration_few_iterations(niter):
    _run(1, 256, 704, 64, 16, 512, torch.bfloat16, niter=niter)


def test_calibration_matches_torch_svd_lowrank():
    """The reference's own call: torch.svd_lowrank on the GPU from the default generator."""
    from dsmezo_b200 import AdapterSet
    R, niter = 16, 3
    mods, bases, A, B, V0, H = make_inputs(1, 384, 1280, 64, R, 768, 9, torch.float32, torch.bfloat16)
    aset = AdapterSet(mods, bases, R, R, copy_dtype=torch.float32, act_dtype=torch.bfloat16, device=DEV)
    for b in range(len(bases)):
        aset.H(b).copy_(H[b])
    torch.cuda.manual_seed(77)
    want = [torch.svd_lowrank(h.to(DEV).float(), q=R, niter=niter)[2].cpu() for h in H]
    end = torch.cuda.default_generators[torch.cuda.current_device()].get_offset()
    torch.cuda.manual_seed(77)
    aset.calibrate(niter=niter)
    torch.cuda.synchronize()
    assert torch.cuda.default_generators[torch.cuda.current_device()].get_offset() == end
    for b, Vt in enumerate(want):
        sine = ref.subspace_sine(aset.V(b).cpu(), Vt)
        assert sine <= SINE_TORCH, f"basis {b}: sine vs torch.svd_lowrank {sine:.2e}"


def test_calibration_then_step_runs():
    """A calibrated set steps on: the power iteration keeps the calibrated subspace's
    leading directions (its bf16 split is rebuilt after the rotation)."""
    aset, bases, H = _run(1, 256, 704, 64, 16, 512, torch.bfloat16)
    before = [aset.V(b).clone() for b in range(len(bases))]
    aset.power_iteration(1)
    torch.cuda.synchronize()
    assert aset.device_error() == 0
    for b in range(len(bases)):
        exp = ref.fused_power_iter(H[b].float(), before[b].cpu(), 1)
        assert ref.subspace_sine(aset.V(b).cpu(), exp) <= 1e-4
