"""The tensor-core power iteration's reuse of the previous iteration's bf16 split of the
bases (DSMZ_PI_BASIS_UNCHANGED): when the basis arena was not written since the last power
iteration, the second call must give bit-identical bases to a call that recomputes the
split, and a write to the basis through torch must force the recomputation."""
import pytest
import torch

from step_harness import make_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _set(seed):
    from dsmezo_b200 import AdapterSet
    mods, bases, A, B, V0, H = make_inputs(1, 256, 704, 64, 16, 512, seed, torch.bfloat16, torch.bfloat16)
    aset = AdapterSet(mods, bases, 16, 16, copy_dtype=torch.bfloat16, act_dtype=torch.bfloat16, device=DEV)
    for i in range(len(mods)):
        aset.A(i).copy_(A[i])
        aset.B(i).copy_(B[i])
    for b in range(len(bases)):
        aset.V(b).copy_(V0[b])
        aset.H(b).copy_(H[b])
    return aset, V0


def test_split_reuse_matches_recompute():
    a, _ = _set(11)
    b, _ = _set(11)
    if not a.uses_tensor_cores:
        pytest.skip("power iteration on CUDA cores: no bf16 split")
    a.power_iteration(3)
    b.power_iteration(3)
    n0a, n0b = a.launches, b.launches
    a.power_iteration(3)                      # basis untouched: split reused
    b.V_arena.add_(0.0)                       # a torch write (same values): split recomputed
    b.power_iteration(3)
    torch.cuda.synchronize()
    assert a.device_error() == 0 and b.device_error() == 0
    assert a.launches - n0a == (b.launches - n0b) - 1
    assert torch.equal(a.V_arena, b.V_arena)


def test_basis_write_forces_split():
    a, V0 = _set(12)
    c, _ = _set(12)
    if not a.uses_tensor_cores:
        pytest.skip("power iteration on CUDA cores: no bf16 split")
    a.power_iteration(2)
    for bi in range(len(V0)):                 # restart from the initial bases through torch
        a.V(bi).copy_(V0[bi])
    a.power_iteration(2)
    c.power_iteration(2)
    torch.cuda.synchronize()
    assert torch.equal(a.V_arena, c.V_arena)
