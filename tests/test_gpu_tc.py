"""The tcgen05 power iteration (bf16 hi/lo operands, fp32 TMEM accumulation) against the
exact (fp64) reference algorithm, against the CUDA-core path, and its error word."""
import pytest
import torch

from oracle import reference_ops as ref
from step_harness import make_inputs, rel

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("T,D,R", [(4096, 3584, 64), (4096, 18944, 64), (2048, 1536, 16), (8192, 512, 128),
                                   (130, 200, 16), (1000, 64, 16), (64, 4096, 32)])
def test_tc_power_iter_dropin(T, D, R):
    from dsmezo_b200 import kernels as K
    g = torch.Generator().manual_seed(T * 3 + D + R)
    scale = torch.exp(torch.randn(D, generator=g))
    H = (torch.randn(T, D, generator=g) * scale).to(torch.bfloat16)
    V0 = torch.linalg.qr(torch.randn(D, R, generator=g))[0]
    V = K.fused_power_iter(H.to(DEV), V0.to(DEV), 3, ref.FLT_MIN)
    want = ref.fused_power_iter(H.double(), V0.double(), 3, ref.FLT_MIN, torch.float64)
    torch.cuda.synchronize()
    assert ref.subspace_sine(V.cpu(), want) < 1e-3       # gate; measured ~1e-5
    assert float((V.cpu().double().T @ V.cpu().double() - torch.eye(R, dtype=torch.float64)).abs().max()) < 1e-5


def _set(tc, rank, seed=4):
    from dsmezo_b200 import AdapterSet
    mods, bases, A, B, V0, H = make_inputs(1, 512, 1536, 128, rank, 384, seed, torch.bfloat16, torch.bfloat16)
    aset = AdapterSet(mods, bases, rank, rank, copy_dtype=torch.bfloat16, act_dtype=torch.bfloat16, device=DEV,
                      tensor_core_power_iter=tc)
    for b in range(len(bases)):
        aset.V(b).copy_(V0[b])
        aset.H(b).copy_(H[b])
    return aset, H, V0


@pytest.mark.parametrize("rank", [16, 64])
def test_tc_grouped_matches_cuda_core_path(rank):
    a_tc, H, V0 = _set(True, rank)
    a_sc, _, _ = _set(False, rank)
    assert a_tc.uses_tensor_cores and not a_sc.uses_tensor_cores
    a_tc.power_iteration(3)
    a_sc.power_iteration(3)
    torch.cuda.synchronize()
    assert a_tc.device_error() == 0
    for b in range(len(H)):
        want = ref.fused_power_iter(H[b].double(), V0[b].double(), 3, ref.FLT_MIN, torch.float64)
        s_tc = ref.subspace_sine(a_tc.V(b).cpu(), want)
        s_sc = ref.subspace_sine(a_sc.V(b).cpu(), want)
        assert s_tc < 1e-3 and s_sc < 1e-4
        assert rel(a_tc.V(b), a_sc.V(b)) < 1e-3


def _pass_set(mods, bases, V0, H, rank, single):
    from dsmezo_b200 import AdapterSet
    aset = AdapterSet(mods, bases, rank, rank, copy_dtype=torch.bfloat16, act_dtype=torch.bfloat16, device=DEV,
                      single_pass_power_iter=single)
    for b in range(len(bases)):
        aset.V(b).copy_(V0[b])
        aset.H(b).copy_(H[b])
    return aset


@pytest.mark.parametrize("layers,hidden,inter,kv,rank,tokens", [
    (1, 512, 1536, 128, 16, 384),     # a partial 256-token tile; no split Y tiles
    (1, 512, 1536, 128, 64, 512),
    (2, 200, 520, 40, 16, 300),       # D not a multiple of 64, ragged tokens
    (1, 3584, 18944, 512, 64, 4096),  # one Qwen2.5-7B-shaped layer: split Y tiles (3 and 15 splits)
])
def test_single_pass_matches_two_pass_and_exact(layers, hidden, inter, kv, rank, tokens):
    """The single-pass power iteration (each activation read from HBM once per iteration) gives
    the bases of the two-product path and of the exact algorithm, and is deterministic."""
    mods, bases, A, B, V0, H = make_inputs(layers, hidden, inter, kv, rank, tokens, 31 + rank, torch.bfloat16,
                                           torch.bfloat16)
    one = _pass_set(mods, bases, V0, H, rank, True)
    two = _pass_set(mods, bases, V0, H, rank, False)
    assert one.single_pass_power_iter and two.uses_tensor_cores and not two.single_pass_power_iter
    one.power_iteration(3)
    two.power_iteration(3)
    again = _pass_set(mods, bases, V0, H, rank, True)
    again.power_iteration(3)
    torch.cuda.synchronize()
    assert one.device_error() == 0 and again.device_error() == 0 and two.device_error() == 0
    assert torch.equal(one.V_arena, again.V_arena)          # fixed summation order
    for b in range(len(bases)):
        want = ref.fused_power_iter(H[b].double(), V0[b].double(), 3, ref.FLT_MIN, torch.float64)
        s1 = ref.subspace_sine(one.V(b).cpu(), want)
        s2 = ref.subspace_sine(two.V(b).cpu(), want)
        assert s1 < 1e-3 and s1 <= max(2e-5, 3 * s2), (b, s1, s2)   # gate 1e-3; as close as two passes
        Vb = one.V(b).cpu().double()
        assert float((Vb.T @ Vb - torch.eye(rank, dtype=torch.float64)).abs().max()) < 1e-5


def test_tc_path_selection():
    from dsmezo_b200 import AdapterSet, transformer_adapter_shapes
    mods, bases = transformer_adapter_shapes(1, 96, 200, 24, 64)
    fp32_acts = AdapterSet(mods, bases, 16, 16, act_dtype=torch.float32, device=DEV)
    assert not fp32_acts.uses_tensor_cores          # tcgen05 path takes bf16 activations
    odd_rank = AdapterSet(mods, bases, 12, 12, act_dtype=torch.bfloat16, device=DEV)
    assert not odd_rank.uses_tensor_cores           # N = 2R must be a multiple of 32
