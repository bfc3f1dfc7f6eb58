"""Expert-parallel fused MoE on 2-8 GPUs (skipped with fewer than two GPUs).

Runs tests/ep_gpu_worker.py under torchrun (one rank per GPU): both expert-parallel paths (NCCL
all-to-all, fused NVLink peer memory) must match the CPU oracle on a seeded sample of tokens at
the north_star bar (max_rel <= 1e-2, cos >= 0.9999). Shapes: a small one, a many-expert top-6
one, and the Mixtral layer of BASELINE configs[3] (T=16384, H=4096, F=14336, E=8, top-2)."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("shape", [(4096, 1024, 2048, 8, 2), (2048, 512, 256, 64, 6),
                                   (16384, 4096, 14336, 8, 2)])
def test_ep_matches_oracle(shape):
    n = min(torch.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("needs at least two GPUs")
    while shape[3] % n:
        n //= 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(HERE, "ep_gpu_worker.py"), *map(str, shape)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("EP_OK") == 3, r.stdout
