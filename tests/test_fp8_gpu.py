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


def test_swiglu_fp8():
    from grouped_gemm_opt import _C, quantize_fp8
    x, w, tpe = gemm_inputs([2000, 0, 3000, 77], 256, 1024, seed=2)  # F = 512
    xq, xs = quantize_fp8(x.to(DEV))
    wq, ws = quantize_fp8(w.to(DEV))
    h = _C.grouped_gemm_swiglu_fp8(xq, xs, wq, ws, tpe.to(DEV), 4, True)
    xd = xq.cpu().float() * xs.cpu().unsqueeze(1)
    wd = wq.cpu().float() * ws.cpu().unsqueeze(-1)
    assert_parity(h, oracle.swiglu_gemm(xd, wd, tpe, 4), "swiglu fp8")


def test_fused_moe_fp8():
    """FP8 layer vs the same quantisation steps on the CPU (dequantised operands, fp32 math)."""
    import numpy as np
    from grouped_gemm_opt import fused_moe_fp8, quantize_moe_weights
    g = torch.Generator().manual_seed(9)
    T, H, F, E, k = 512, 512, 1024, 8, 2
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    wgu = (torch.randn(E, 2 * F, H, generator=g) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(E, H, F, generator=g) * 0.02).to(torch.bfloat16)
    qw = quantize_moe_weights(wgu.to(DEV), wd.to(DEV))
    out = fused_moe_fp8(x.to(DEV), logits.to(DEV), qw, k)
    # CPU restatement of the FP8 pipeline
    ids, w, tpe = oracle.route(logits.numpy(), k)
    st, pos = oracle.permute_indices(ids, E)
    xs = x[torch.from_numpy(st).long()]
    xq, xsc = _ref_quant(xs)
    gud = qw.w_gate_up_q.cpu().float() * qw.w_gate_up_scale.cpu().unsqueeze(-1)
    h = oracle.swiglu_gemm(xq.float() * xsc.unsqueeze(1), gud, torch.from_numpy(tpe), E)
    hq, hsc = _ref_quant(h.to(torch.bfloat16))
    dd = qw.w_down_q.cpu().float() * qw.w_down_scale.cpu().unsqueeze(-1)
    y = oracle.segments_gemm(hq.float() * hsc.unsqueeze(1), dd, torch.from_numpy(tpe), E)
    ref = oracle.combine(y.to(torch.bfloat16), w, pos)
    assert_parity(out, ref, "fused moe fp8")
    rel, cos = parity(out, oracle.moe_layer(x, logits, wgu, wd, k, round_to=torch.bfloat16))
    assert cos > 0.995, cos  # vs the bf16 layer: e4m3 quantisation error only


def test_fp8_cfg2_full_size_sampled():
    from grouped_gemm_opt import grouped_gemm_opt_fp8, quantize_fp8
    T, E, K, N = 4096, 8, 4096, 14336
    tpe = torch.full((E,), 512)
    g = torch.Generator(device=DEV).manual_seed(6)
    x = torch.randn(T, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(E, N, K, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    xq, xs = quantize_fp8(x)
    wq, ws = quantize_fp8(w)
    out = grouped_gemm_opt_fp8(xq, xs, wq, ws, tpe.to(DEV))
    rows = torch.arange(3, T, 97)
    ref = []
    for r in rows.tolist():
        e = r // 512
        a = xq[r].float().cpu() * xs[r].cpu()
        b = wq[e].float().cpu() * ws[e].cpu().unsqueeze(1)
        ref.append(b @ a)
    assert_parity(out[rows.to(DEV)], torch.stack(ref), "fp8 cfg2")


@pytest.mark.parametrize("rows,cols", [(37, 14336), (5, 16384), (3, 16400), (64, 1040), (9, 16)])
def test_quantize_bit_exact_row_widths(rows, cols):
    """Both quantiser forms: rows held in registers (cols <= 16384) and the two-pass one."""
    from grouped_gemm_opt import quantize_fp8
    g = torch.Generator().manual_seed(cols)
    x = (torch.randn(rows, cols, generator=g) * torch.logspace(-2, 2, rows).unsqueeze(1)).to(
        torch.bfloat16)
    q, s = quantize_fp8(x.to(DEV))
    rq, rs = _ref_quant(x)
    assert torch.equal(s.cpu(), rs)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))
