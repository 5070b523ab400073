"""GPU parity of the contrastive scoring loss (dsmz_contrastive_loss, via
dsmezo_b200.scoring) against the reference's own _score_contrastive (golden fixture
tests/golden/scoring.pt) and the CPU oracle. Tolerances: 1e-6 relative from fp32 logits
(the kernel's fp32 log-sum-exp against torch's fp32 log_softmax), 1e-12 from logprobs
(fp64 sums in another order); bit-identical between two runs."""
from pathlib import Path

import pytest
import torch

from oracle import reference_ops as ref

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
DEV = "cuda"


@pytest.fixture(scope="module")
def S():
    from dsmezo_b200 import scoring
    return scoring


@pytest.fixture(scope="module")
def cases():
    return torch.load(GOLD / "scoring.pt", weights_only=False)


def rel(a, b):
    return abs(a - b) / max(abs(b), 1e-30)


def test_logits_f32_match_the_reference(S, cases):
    for c in cases:
        for k in ("pos", "neg"):
            got = float(S.contrastive_loss(c[f"rows_{k}"].to(DEV), c["seq_tokens"], c["advantages"],
                                           c["targets"].to(DEV)))
            assert rel(got, c[f"loss_{k}"]) < 1e-6, (k, got, c[f"loss_{k}"])


def test_logprobs_match_the_reference(S, cases):
    for c in cases:
        for k in ("pos", "neg"):
            lp = torch.log_softmax(c[f"rows_{k}"].float(), -1).gather(1, c["targets"].long()[:, None]).flatten()
            got = float(S.contrastive_loss(lp.to(DEV), c["seq_tokens"], c["advantages"]))
            assert rel(got, c[f"loss_{k}"]) < 1e-12, (k, got, c[f"loss_{k}"])


def test_bf16_and_strided_logits(S, cases):
    for c in cases:
        rows = c["rows_pos"].to(torch.bfloat16)
        want = ref.contrastive_loss(rows.float(), c["targets"].tolist(), c["seq_tokens"], c["advantages"])
        got = float(S.contrastive_loss(rows.to(DEV), c["seq_tokens"], c["advantages"], c["targets"].to(DEV)))
        assert rel(got, want) < 1e-6
        # rows inside a wider buffer (row pitch > V: the element path when the pitch is odd)
        wide = torch.zeros(rows.shape[0], rows.shape[1] + 3, dtype=torch.float32)
        wide[:, :rows.shape[1]] = c["rows_pos"]
        view = wide.to(DEV)[:, :rows.shape[1]]
        got = float(S.contrastive_loss(view, c["seq_tokens"], c["advantages"], c["targets"].to(DEV)))
        assert rel(got, c["loss_pos"]) < 1e-6


def test_scoring_vocabulary_size_and_determinism(S):
    # Qwen2.5 vocabulary (152064), four completions of 512 scored tokens, bf16 logits
    g = torch.Generator(device=DEV).manual_seed(5)
    V, lens = 152064, [512, 512, 512, 512]
    rows = (torch.randn(sum(lens), V, generator=g, device=DEV) * 4).to(torch.bfloat16)
    tg = torch.randint(0, V, (sum(lens),), generator=g, device=DEV, dtype=torch.int32)
    adv = [0.75, -0.25, -0.25, -0.25]
    a = S.contrastive_loss(rows, lens, adv, tg)
    b = S.contrastive_loss(rows, lens, adv, tg)
    lp = torch.log_softmax(rows.double(), -1).gather(1, tg.long()[:, None]).flatten()
    want = sum(-adv[i] * float(lp[512 * i:512 * (i + 1)].mean()) for i in range(4))
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert rel(float(a), want) < 1e-6


def test_target_outside_the_vocabulary_gives_nan(S):
    rows = torch.randn(6, 40, device=DEV)
    tg = torch.tensor([1, 2, 3, 40, 5, 6], dtype=torch.int32, device=DEV)
    assert torch.isnan(S.contrastive_loss(rows, [3, 3], [1.0, -1.0], tg)).item()
    tg[3] = 7
    assert not torch.isnan(S.contrastive_loss(rows, [3, 3], [1.0, -1.0], tg)).item()
