"""FP8 (e4m3) path: row quantisation bit-exact against torch's own float8 conversion, and the
kind::f8f6f4 grouped GEMM against the CPU oracle run on the dequantised operands (the same
products, so the bf16 parity bar applies). The FP8 result is also compared with the bf16 GEMM of
the unquantised operands, at FP8's own looser tolerance."""
import pytest
import torch

import grouped_gemm_oracle as oracle
from gpu_util import assert_parity, parity
from inputs import gemm_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _ref_quant(x):
    xf = x.float()
    amax = xf.abs().amax(dim=-1)
    s = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    return (xf / s.unsqueeze(-1)).to(torch.float8_e4m3fn), s


def test_quantize_bit_exact():
    from grouped_gemm_opt import quantize_fp8
    g = torch.Generator().manual_seed(0)
    x = (torch.randn(333, 1024, generator=g) * torch.logspace(-3, 3, 333).unsqueeze(1)).to(
        torch.bfloat16)
    x[5] = 0
    q, s = quantize_fp8(x.to(DEV))
    rq, rs = _ref_quant(x)
    assert torch.equal(s.cpu(), rs)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))


@pytest.mark.parametrize("tc", [1, 3, 4])
@pytest.mark.parametrize("counts,k,n", [([32] * 8, 512, 1024), ([1, 7, 8, 127, 128, 129, 0], 256, 384),
                                        ([700, 300, 1100, 20], 1024, 2048)])
def test_fp8_grouped_gemm(tc, counts, k, n):
    from grouped_gemm_opt import grouped_gemm_opt_fp8, quantize_fp8
    x, w, tpe = gemm_inputs(counts, k, n, seed=k + tc)
    xq, xs = quantize_fp8(x.to(DEV))
    wq, ws = quantize_fp8(w.to(DEV))  # per output channel: scale [E, N]
    out = grouped_gemm_opt_fp8(xq, xs, wq, ws, tpe.to(DEV), tc)
    assert out.dtype == torch.bfloat16 and out.shape == (x.size(0), n)
    xd = xq.cpu().float() * xs.cpu().unsqueeze(1)
    wd = wq.cpu().float() * ws.cpu().unsqueeze(-1)
    assert_parity(out, oracle.sequential_gemm(xd, wd, tpe), f"fp8 tc={tc}")
    rel, cos = parity(out, oracle.sequential_gemm(x, w, tpe))
    assert rel < 0.1 and cos > 0.998, (rel, cos)  # e4m3 quantisation error vs the bf16 GEMM
