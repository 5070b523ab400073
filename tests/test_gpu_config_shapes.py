"""Step parity at the shapes of the benchmark configurations, against the fp32 and fp64
oracles with the CUDA-generator draws (two-oracle criterion of test_gpu_step.py):

* one full Qwen2.5-7B-shaped layer (hidden 3584, intermediate 18944, k/v 512, rank 64,
  4096 tokens, bf16 inputs, cubic schedule), two steps;
* the whole Qwen2.5-1.5B-shaped set (28 layers, hidden 1536, intermediate 8960, k/v 256,
  rank 16, 2048 tokens, bf16 inputs, quintic schedule), two steps;
* one Llama-3-70B-shaped layer (hidden 8192, intermediate 28672, k/v 1024, rank 128, 8192
  tokens, bf16 inputs, cubic schedule), one step.

The masters are fp32 and each step checks that they moved by -eta * X (test_gpu_step.py)."""
import pytest
import torch

from test_gpu_step import _run_case

pytestmark = pytest.mark.gpu


def test_qwen7b_layer_two_steps():
    _run_case(1, 3584, 18944, 512, 64, 4096, seed=2, copy_dtype=torch.bfloat16, act_dtype=torch.bfloat16, steps=2,
              total_steps=1000, schedule="cubic")


def test_qwen15b_set_two_steps():
    _run_case(28, 1536, 8960, 256, 16, 2048, seed=1, copy_dtype=torch.bfloat16, act_dtype=torch.bfloat16, steps=2,
              total_steps=1000, schedule="quintic")


def test_llama70b_layer_rank128_one_step():
    _run_case(1, 8192, 28672, 1024, 128, 8192, seed=3, copy_dtype=torch.bfloat16, act_dtype=torch.bfloat16, steps=1,
              total_steps=1000, schedule="cubic")
