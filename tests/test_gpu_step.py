"""GPU parity of the grouped optimizer step (AdapterSet + ZOController) against the oracle's
replay of the reference controller with the same CUDA-generator draws.

Covers: power iteration of every unique activation, Zc_B / Zc_A regeneration from the
Philox stream (checked bit-exactly through the generator offset), AGZO z, pos/neg, the
Kalman predict/observe, ZO-Muon NS and the cosine eta; two consecutive steps.
"""
import math

import pytest
import torch

from oracle import reference_ops as ref
from step_harness import cuda_draws, make_inputs, oracle_state, rel

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run_case(layers, hidden, inter, kv, rank, tokens, seed, factor_dtype, act_dtype, steps=2, total_steps=100,
              eps=1e-3, schedule="cubic", warm_mu=False):
    from dsmezo_b200 import AdapterSet, ZOController
    mods, bases, A, B, V0, H = make_inputs(layers, hidden, inter, kv, rank, tokens, seed, factor_dtype, act_dtype)
    aset = AdapterSet(mods, bases, rank, rank, factor_dtype=factor_dtype, act_dtype=act_dtype, device=DEV,
                      keep_ns_output=True)
    g = torch.Generator().manual_seed(seed + 1)
    mu0 = [(torch.randn(m.d_out, rank, generator=g), torch.randn(rank, m.d_in, generator=g)) if warm_mu else None
           for m in mods]
    for i in range(len(mods)):
        aset.A(i).copy_(A[i])
        aset.B(i).copy_(B[i])
        if warm_mu:
            aset.A(i, aset.mu).copy_(mu0[i][0])
            aset.B(i, aset.mu).copy_(mu0[i][1])
    aset.var.fill_(eps ** 2)
    for b in range(len(bases)):
        aset.V(b).copy_(V0[b])
        aset.H(b).copy_(H[b])
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    ctl = ZOController(aset, eps, total_steps, gen, schedule=schedule)
    st = oracle_state(mods, [a.float() for a in A], [b.float() for b in B], V0, eps, total_steps,
                      mu=mu0 if warm_mu else None, schedule=ref.get_schedule(schedule))
    acts = [h.float() for h in H]
    for _ in range(steps):
        off0 = gen.get_offset()
        ctl.perturb()
        draws, off_end = cuda_draws(mods, rank, rank, seed, off0, DEV)
        assert gen.get_offset() == off_end           # generator advanced exactly like the reference
        st.step_count += 1
        perts = ref.perturb_phase(st, acts, draws, 3)
        torch.cuda.synchronize()
        for b in range(len(bases)):
            assert ref.subspace_sine(aset.V(b).cpu(), st.bases[b]) < 1e-4
        for i, m in enumerate(st.modules):
            zA, zB = perts[i]
            assert rel(aset.A(i, aset.z), zA) < 1e-4, (i, "z_A")
            assert rel(aset.B(i, aset.z), zB) < 1e-4, (i, "z_B")
            if factor_dtype == torch.float32:
                assert rel(aset.A(i, aset.pos) - aset.A(i), m.pos_A - m.A) < 1e-4
                assert rel(aset.B(i, aset.neg) - aset.B(i), m.neg_B - m.B) < 1e-4
        dd = 3.7 * (st.step_count + 1)
        ref.update_phase(st, perts, dd)
        ctl.update(dd)
        torch.cuda.synchronize()
        assert math.isclose(ctl.eta, st.eta, rel_tol=1e-12)
        tol = 1e-4 if factor_dtype == torch.float32 else 2e-2
        for i, m in enumerate(st.modules):
            assert rel(aset.A(i, aset.mu), m.mu_A) < 1e-4, (i, "mu_A")
            assert rel(aset.B(i, aset.mu), m.mu_B) < 1e-4, (i, "mu_B")
            assert rel(aset.A(i, aset.var), m.var_A) < 1e-4, (i, "var_A")
            assert rel(aset.B(i, aset.var), m.var_B) < 1e-4, (i, "var_B")
            assert rel(aset.A(i, aset.scratch), m.scratch_A) < 1e-4 * (1 if factor_dtype == torch.float32 else 10)
            assert rel(aset.B(i, aset.scratch), m.scratch_B) < 1e-4 * (1 if factor_dtype == torch.float32 else 10)
            if factor_dtype == torch.float32:
                a0 = A[i].float()
                assert rel(aset.A(i).cpu() - a0, m.A - a0) < tol
            # keep the oracle on the stored factors (bf16 rounding of the param happens on store)
            m.A.copy_(aset.A(i).float().cpu())
            m.B.copy_(aset.B(i).float().cpu())
            A[i] = aset.A(i).float().cpu().clone()
    return aset


def test_step_toy_shape_fp32():
    """The toy set: 4 layers, hidden 512, intermediate 1408, k/v 128, rank 8, 256 tokens."""
    _run_case(4, 512, 1408, 128, 8, 256, seed=0, factor_dtype=torch.float32, act_dtype=torch.float32)


def test_step_odd_shapes_warm_momentum():
    _run_case(2, 96, 200, 24, 12, 72, seed=5, factor_dtype=torch.float32, act_dtype=torch.float32, warm_mu=True)


def test_step_rank64_bf16_quintic():
    _run_case(1, 512, 1536, 128, 64, 512, seed=2, factor_dtype=torch.bfloat16, act_dtype=torch.bfloat16,
              schedule="quintic")


def test_step_rank128_bf16():
    _run_case(1, 384, 1024, 128, 128, 256, seed=3, factor_dtype=torch.bfloat16, act_dtype=torch.bfloat16, steps=1)
