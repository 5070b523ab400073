"""Many-direction SPSA on the GPU against the oracle's restatement (no reference
counterpart: the reference observes one direction per step). Direction k must take
exactly the draws of the k-th of K successive one-direction steps, its z and +/- copies
must match the one-direction perturbation, and the joint Kalman update plus ZO-Muon
must match the oracle (two-oracle criterion as in the one-direction step test)."""
import math

import pytest
import torch

from oracle import reference_ops as ref
from step_harness import cuda_draws, make_inputs, oracle_state, rel

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {"z": 2e-5, "mu": 1e-5, "var": 1e-6, "X": 1e-5}
TC = 10.0


def close(name, ours, o32, o64, what, scale):
    d_ours, d_ref = rel(ours, o64), rel(o32, o64)
    assert d_ours <= max(TOL[name] * scale, 2.0 * d_ref), f"{what}: |ours-exact| {d_ours:.2e}, |ref32-exact| {d_ref:.2e}"


@pytest.mark.parametrize("K,fdt", [(3, torch.bfloat16), (2, torch.float32), (16, torch.bfloat16)])
def test_directions_step(K, fdt):
    from dsmezo_b200 import AdapterSet, ZOController
    layers, hidden, inter, kv, rank, tokens, seed = 1, 384, 1280, 64, 16, 256, 11
    mods, bases, A, B, V0, H = make_inputs(layers, hidden, inter, kv, rank, tokens, seed, fdt, torch.bfloat16)
    aset = AdapterSet(mods, bases, rank, rank, copy_dtype=fdt, act_dtype=torch.bfloat16, device=DEV,
                      keep_ns_output=True, directions=K)
    scale = TC if aset.uses_tensor_cores else 1.0
    for i in range(len(mods)):
        aset.A(i).copy_(A[i])
        aset.B(i).copy_(B[i])
    eps = 1e-3
    aset.var.fill_(eps ** 2)
    for b in range(len(bases)):
        aset.V(b).copy_(V0[b])
        aset.H(b).copy_(H[b])
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    ctl = ZOController(aset, eps, 100, gen, schedule="quintic")
    st = {dt: oracle_state(mods, A, B, V0, eps, 100, schedule=ref.get_schedule("quintic"), dtype=dt)
          for dt in (torch.float32, torch.float64)}
    acts = {dt: [h.to(dt) for h in H] for dt in st}
    inc1 = aset.rng_increment // K
    for step in range(2):
        off0 = gen.get_offset()
        ctl.perturb()
        assert gen.get_offset() == off0 + K * inc1
        draws_dirs = []
        for k in range(K):
            d, end = cuda_draws(mods, rank, rank, seed, off0 + k * inc1, DEV)
            assert end == off0 + (k + 1) * inc1
            draws_dirs.append(d)
        perts = {}
        for dt, s in st.items():
            s.step_count += 1
            perts[dt] = ref.perturb_phase_directions(s, acts[dt], draws_dirs, 3)
        torch.cuda.synchronize()
        for k in range(K):
            for i in range(len(mods)):
                (a32, b32), (a64, b64) = perts[torch.float32][k][i], perts[torch.float64][k][i]
                close("z", aset.A(i, aset.z_dir(k)), a32, a64, f"step {step} dir {k} module {i} z_A", scale)
                close("z", aset.B(i, aset.z_dir(k)), b32, b64, f"step {step} dir {k} module {i} z_B", scale)
                # the +/- copies are the factor plus / minus our own z, rounded to the factor dtype
                zA = aset.A(i, aset.z_dir(k))
                p = aset.A(i).float()
                assert torch.equal(aset.A(i, aset.pos_dir(k)), (p + zA).to(fdt))
                assert torch.equal(aset.A(i, aset.neg_dir(k)), (p - zA).to(fdt))
        g = torch.Generator().manual_seed(100 + step)
        rewards = torch.bernoulli(torch.full((K, 8), 0.4), generator=g)
        dds = ref.rloo_direction_scalars(rewards, eps)
        for dt, s in st.items():
            ref.update_phase_directions(s, perts[dt], dds)
        ctl.update(dds)
        torch.cuda.synchronize()
        assert aset.device_error() == 0
        o32, o64 = st[torch.float32], st[torch.float64]
        assert math.isclose(ctl.eta, o64.eta, rel_tol=1e-12)
        for i in range(len(mods)):
            m32, m64 = o32.modules[i], o64.modules[i]
            for side in ("A", "B"):
                view = aset.A if side == "A" else aset.B
                close("mu", view(i, aset.mu), getattr(m32, "mu_" + side), getattr(m64, "mu_" + side),
                      f"step {step} module {i} mu_{side}", scale)
                close("var", view(i, aset.var), getattr(m32, "var_" + side), getattr(m64, "var_" + side),
                      f"step {step} module {i} var_{side}", scale)
                close("X", view(i, aset.scratch), getattr(m32, "scratch_" + side), getattr(m64, "scratch_" + side),
                      f"step {step} module {i} NS output {side}", scale)
                p = view(i).float().cpu()
                getattr(m32, side).copy_(p)
                getattr(m64, side).copy_(p.double())
