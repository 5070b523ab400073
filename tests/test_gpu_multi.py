"""Layer-sharded step on 2 GPUs (NCCL) against the same step on one GPU. Skipped when the
machine shows fewer than two GPUs."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("factor_gather,perturb", [("copy-engine", "tensor-cores"), ("fused", "tensor-cores"),
                                                    ("nccl", "tensor-cores"), ("copy-engine", "cuda-cores")])
def test_two_rank_step_matches_one_gpu(factor_gather, perturb):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", DSMZ_FACTOR_GATHER=factor_gather, DSMZ_PERTURB=perturb)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(HERE, "multi_gpu_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "MULTI_OK" in r.stdout
    # two GPUs of one node: the +/- copies are gathered by the perturbation's peer stores
    # (either perturbation kernel), the factors by the mode asked for
    assert f"FUSED_GATHER True {factor_gather}" in r.stdout, r.stdout[-2000:]
