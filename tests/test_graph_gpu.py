"""The grouped GEMM and the single-GPU MoE layer replay correctly from a CUDA graph: counts stay
on the device, the work-stealing counters reset themselves at the end of every launch, and no
host synchronisation happens inside the calls."""
import pytest
import torch

import grouped_gemm_oracle as oracle
from gpu_util import assert_parity
from inputs import gemm_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_grouped_gemm_graph_replay():
    import grouped_gemm_opt as ggo
    x, w, tpe = gemm_inputs([300, 0, 513, 17, 256], 256, 512, seed=3)
    xd, wd, td = x.to(DEV), w.to(DEV), tpe.to(DEV)
    ggo.grouped_gemm_opt(xd, wd, td)  # warm-up outside capture (one-time set-up)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ggo.grouped_gemm_opt(xd, wd, td)
    for i in range(3):
        xd.copy_((x.float() * (i + 1)).to(torch.bfloat16))
        g.replay()
        torch.cuda.synchronize()
        ref = oracle.sequential_gemm((x.float() * (i + 1)).to(torch.bfloat16), w, tpe)
        assert_parity(out, ref, f"graph replay {i}")
    ggo.check_device_errors(0)


def test_fused_moe_graph_replay():
    import grouped_gemm_opt as ggo
    gen = torch.Generator().manual_seed(1)
    T, H, F, E, k = 256, 256, 512, 8, 2
    x = torch.randn(T, H, generator=gen).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=gen)
    wgu = (torch.randn(E, 2 * F, H, generator=gen) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(E, H, F, generator=gen) * 0.02).to(torch.bfloat16)
    xd, ld, gud, dd = x.to(DEV), logits.to(DEV), wgu.to(DEV), wd.to(DEV)
    ggo.fused_moe(xd, ld, gud, dd, k)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ggo.fused_moe(xd, ld, gud, dd, k)
    lg2 = torch.randn(T, E, generator=gen)
    ld.copy_(lg2)  # new routing, same shapes
    g.replay()
    torch.cuda.synchronize()
    assert_parity(out, oracle.moe_layer(x, lg2, wgu, wd, k, round_to=torch.bfloat16), "moe graph")
