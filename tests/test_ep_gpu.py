"""Expert-parallel fused MoE over NCCL on 2-8 GPUs (skipped with fewer than two GPUs).

Runs tests/ep_gpu_worker.py under torchrun (one rank per GPU) and requires every rank's EP
output to match the single-GPU layer on the same tokens."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("shape", [(4096, 1024, 2048, 8, 2), (2048, 512, 256, 64, 6)])
def test_ep_nccl_matches_single_gpu(shape):
    n = min(torch.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("needs at least two GPUs")
    while shape[3] % n:
        n //= 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(HERE, "ep_gpu_worker.py"), *map(str, shape)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("EP_OK") == n, r.stdout
