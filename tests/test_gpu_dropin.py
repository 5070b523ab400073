"""GPU parity of the four drop-in ops (dsmezo_b200.kernels) against the reference's golden
vectors and the CPU oracle, through the C ABI. Tolerances: Newton-Schulz output 1e-5
relative Frobenius (fp32) / 2e-2 (bf16 factors); power-iteration subspace sine 1e-3
(checked tighter, 1e-4); AGZO z 1e-5; dual perturb bit-exact."""
from pathlib import Path

import pytest
import torch

from oracle import reference_ops as ref
from step_harness import rel

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
FLOOR = ref.FLT_MIN
DEV = "cuda"


@pytest.fixture(scope="module")
def K():
    from dsmezo_b200 import kernels
    return kernels


@pytest.fixture(scope="module")
def kern():
    return torch.load(GOLD / "kernels.pt", weights_only=False)


@pytest.mark.parametrize("name", ["tall_1408x8", "tall_200x16", "tall_16x16", "wide_8x512", "wide_16x1000",
                                  "wide_4x37"])
def test_zo_muon_golden(K, kern, name):
    c = kern[f"muon_{name}"]
    param = c["param_in"].to(DEV)
    scratch = torch.zeros_like(param)
    K.zo_muon_update(param, c["buf"].to(DEV), scratch, c["eta"], FLOOR)
    torch.cuda.synchronize()
    assert rel(scratch, c["scratch_out"]) < 1e-5
    # param is ~1 and the step ~1e-4, so compare values (ulp level), not differences
    assert rel(param, c["param_out"]) < 1e-6


@pytest.mark.parametrize("M,N", [(3584, 64), (64, 3584), (512, 64), (64, 64), (300, 5), (12, 700), (2048, 128),
                                 (128, 1000), (1, 1), (33, 48)])
@pytest.mark.parametrize("sched", ["cubic", "quintic"])
def test_zo_muon_shapes(K, M, N, sched):
    g = torch.Generator().manual_seed(M * 7919 + N)
    param = torch.randn(M, N, generator=g)
    buf = torch.randn(M, N, generator=g)
    p_d, s_d = param.to(DEV), torch.zeros(M, N, device=DEV)
    K.zo_muon_update(p_d, buf.to(DEV), s_d, 0.01, FLOOR, schedule=sched)
    X = ref.ns_orthogonalize(buf.double(), FLOOR, ref.get_schedule(sched)).double()  # fp64 X-space truth
    torch.cuda.synchronize()
    assert rel(s_d, X) < 1e-5
    assert rel(p_d, param.double() - 0.01 * X) < 1e-6


def test_zo_muon_strided_and_bf16(K):
    g = torch.Generator().manual_seed(3)
    base = torch.randn(200, 24, generator=g)
    buf = torch.randn(200, 24, generator=g)
    # transposed view (non-unit column stride) for all three tensors
    pT = base.t().contiguous().to(DEV).t()
    bT = buf.t().contiguous().to(DEV).t()
    sT = torch.zeros(24, 200, device=DEV).t()
    K.zo_muon_update(pT, bT, sT, 0.05, FLOOR)
    X = ref.ns_orthogonalize(buf.double(), FLOOR).double()
    torch.cuda.synchronize()
    assert rel(sT, X) < 1e-5
    # mismatched strides between param and buf are handled by the shim
    p2 = base.to(DEV)
    s2 = torch.zeros(200, 24, device=DEV)
    K.zo_muon_update(p2, bT, s2, 0.05, FLOOR)
    assert rel(s2, X) < 1e-5
    # bf16 factor: fp32 arithmetic, one rounding on store
    pb = base.to(torch.bfloat16).to(DEV)
    sb = torch.zeros(200, 24, device=DEV)
    K.zo_muon_update(pb, buf.to(DEV), sb, 0.05, FLOOR)
    want = (base.to(torch.bfloat16).float() - 0.05 * X.float()).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert rel(sb, X) < 1e-5
    assert rel(pb.float(), want.float()) < 2e-2
    assert (pb.cpu().float() - want.float()).abs().max() <= 2 ** -7 * want.float().abs().max()


@pytest.mark.parametrize("name", ["t256_d512_r8", "t64_d200_r8", "t130_d96_r16", "t32_d48_r5"])
def test_power_iter_golden(K, kern, name):
    c = kern[f"pi_{name}"]
    V = K.fused_power_iter(c["H"].to(DEV), c["V0"].to(DEV), c["iters"], FLOOR)
    torch.cuda.synchronize()
    assert ref.subspace_sine(V.cpu(), c["V"]) < 1e-4
    assert rel(V, c["V"]) < 1e-3       # same basis, not only the same span


@pytest.mark.parametrize("T,D,R,dt", [(4096, 3584, 64, torch.bfloat16), (2048, 1536, 16, torch.bfloat16),
                                      (300, 1000, 12, torch.float32), (8192, 512, 128, torch.bfloat16)])
def test_power_iter_shapes(K, T, D, R, dt):
    g = torch.Generator().manual_seed(T + D + R)
    scale = torch.exp(torch.randn(D, generator=g))
    H = (torch.randn(T, D, generator=g) * scale).to(dt)
    V0 = torch.linalg.qr(torch.randn(D, R, generator=g))[0]
    V = K.fused_power_iter(H.to(DEV), V0.to(DEV), 3, FLOOR)
    want = ref.fused_power_iter(H.double(), V0.double(), 3, FLOOR)
    torch.cuda.synchronize()
    assert ref.subspace_sine(V.cpu(), want) < 1e-3
    assert float((V.cpu().double().T @ V.cpu().double() - torch.eye(R, dtype=torch.float64)).abs().max()) < 1e-5


@pytest.mark.parametrize("name", ["q_128x8x512_rc8", "o_300x8x200_rc4", "k_64x4x96_rc8", "g_704x16x256_rc16"])
def test_agzo_golden(K, kern, name):
    c = kern[f"agzo_{name}"]
    z_A, z_B = K.fused_agzo_perturbation(c["B"].to(DEV), c["V"].to(DEV), c["zcB"].to(DEV), c["zcA"].to(DEV),
                                         c["eps"], FLOOR)
    torch.cuda.synchronize()
    assert rel(z_B, c["z_B"]) < 1e-5
    assert rel(z_A, c["z_A"]) < 1e-5


@pytest.mark.parametrize("R,d_in,RC,d_out", [(64, 3000, 64, 700), (128, 2000, 128, 500), (96, 800, 128, 200),
                                              (128, 1500, 96, 300), (100, 600, 100, 150)])
def test_agzo_strided_and_contiguity(K, R, d_in, RC, d_out):
    """Square and rectangular B V; past 64 x 64 the QR keeps G and R^-1 in the workspace (or,
    for a rank that is not a multiple of 8, runs modified Gram-Schmidt)."""
    g = torch.Generator().manual_seed(11)
    B = torch.randn(d_in, R, generator=g).t()         # strided view
    V = torch.linalg.qr(torch.randn(d_in, RC, generator=g))[0]
    zcB = torch.randn(R, RC, generator=g)
    zcA = torch.randn(d_out, min(R, RC), generator=g)
    z_A, z_B = K.fused_agzo_perturbation(B.to(DEV), V.to(DEV), zcB.to(DEV), zcA.to(DEV), 1e-3, FLOOR)
    # compare with the exact (fp64) algorithm; fp32 MGS carries ~1e-7*cond noise
    wA, wB = ref.fused_agzo_perturbation(B.contiguous(), V, zcB, zcA, 1e-3, FLOOR, dtype=torch.float64)
    torch.cuda.synchronize()
    assert rel(z_B, wB) < 1e-5 and rel(z_A, wA) < 1e-5
    with pytest.raises(AssertionError):
        K.fused_agzo_perturbation(B.to(DEV), V.to(DEV), zcB.to(DEV).t(), zcA.to(DEV), 1e-3, FLOOR)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_dual(K, kern, dt):
    c = kern["dual"]
    base = c["base"].to(dt).to(DEV)
    z = c["z"].to(DEV)
    pos, neg = torch.empty_like(base), torch.empty_like(base)
    K.fused_perturb_dual(base, z, pos, neg)
    torch.cuda.synchronize()
    want_pos = (base.float().cpu() + c["z"]).to(dt)
    want_neg = (base.float().cpu() - c["z"]).to(dt)
    assert torch.equal(pos.cpu(), want_pos) and torch.equal(neg.cpu(), want_neg)
    if dt == torch.float32:
        assert torch.equal(pos.cpu(), c["pos"]) and torch.equal(neg.cpu(), c["neg"])


def test_cpu_tensors_raise(K):
    with pytest.raises(ValueError):
        K.fused_perturb_dual(torch.zeros(4), torch.zeros(4), torch.zeros(4), torch.zeros(4))
