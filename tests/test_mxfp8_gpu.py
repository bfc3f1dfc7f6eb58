"""MXFP8 path (block-scaled e4m3, OCP MX): the quantiser bit-exact against the CPU restatement
(e4m3 bytes and UE8M0 scales in the 128x4 blocked layout), and the kind::mxf8f6f4.block_scale
grouped GEMMs against the CPU oracle run on the dequantised operands (the same products, so the
bf16 parity bar applies). Results are also compared with the bf16 GEMM of the unquantised
operands at MX's own looser tolerance."""
import numpy as np
import pytest
import torch

import grouped_gemm_oracle as oracle
from gpu_util import assert_parity, parity
from inputs import gemm_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _deq(q, sf, counts, k):
    return oracle.mx_dequantize(q.cpu().view(torch.uint8).reshape(-1, k), sf.cpu().numpy(),
                                counts, k)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_quantize_mxfp8_bit_exact(dtype):
    from grouped_gemm_opt import quantize_mxfp8
    g = torch.Generator().manual_seed(0)
    counts = [100, 0, 300, 1, 129, 0]
    T, K = sum(counts), 512
    scale = torch.logspace(-4, 4, T) if dtype == torch.bfloat16 else torch.logspace(-2, 2, T)
    x = (torch.randn(T, K, generator=g) * scale.unsqueeze(1)).to(dtype)
    x[7] = 0
    x[8, :64] = 0
    q, sf = quantize_mxfp8(x.to(DEV), torch.tensor(counts).to(DEV))
    rq, rsf = oracle.mx_quantize(x, counts)
    assert torch.equal(q.cpu().view(torch.uint8), rq)
    assert np.array_equal(sf.cpu().numpy(), rsf)


def test_quantize_mxfp8_weights_bit_exact():
    from grouped_gemm_opt import quantize_mxfp8
    g = torch.Generator().manual_seed(1)
    w = (torch.randn(3, 200, 256, generator=g) * 0.02).to(torch.bfloat16)
    q, sf = quantize_mxfp8(w.to(DEV))
    rq, rsf = oracle.mx_quantize(w.view(-1, 256), [200] * 3)
    assert torch.equal(q.cpu().view(torch.uint8).view(-1, 256), rq)
    assert np.array_equal(sf.cpu().numpy(), rsf)


@pytest.mark.parametrize("sort_by_m", [True, False])
@pytest.mark.parametrize("counts,k,n", [
    ([32] * 8, 512, 1024),
    ([1, 7, 8, 127, 128, 129, 255, 256, 257, 0], 256, 384),
    ([700, 300, 1100, 20], 1024, 2048),
    ([5], 128, 200),          # ragged last column tile (its B scales start 64 rows into a block)
    ([0, 0, 300, 0], 384, 1000),
])
def test_mxfp8_grouped_gemm(counts, k, n, sort_by_m):
    from grouped_gemm_opt import grouped_gemm_opt_mxfp8, quantize_mxfp8
    x, w, tpe = gemm_inputs(counts, k, n, seed=k + n)
    E = len(counts)
    xq, xs = quantize_mxfp8(x.to(DEV), tpe.to(DEV))
    wq, ws = quantize_mxfp8(w.to(DEV))
    out = grouped_gemm_opt_mxfp8(xq, xs, wq, ws, tpe.to(DEV), sort_by_m=sort_by_m)
    assert out.dtype == torch.bfloat16 and out.shape == (x.size(0), n)
    xd = _deq(xq, xs, counts, k)
    wd = _deq(wq, ws, [n] * E, k).view(E, n, k)
    assert_parity(out, oracle.sequential_gemm(xd, wd, tpe), f"mxfp8 {counts[:4]} k={k} n={n}")
    rel, cos = parity(out, oracle.sequential_gemm(x, w, tpe))
    assert rel < 0.1 and cos > 0.998, (rel, cos)  # MX quantisation error vs the bf16 GEMM


def test_mxfp8_segments_rank_major():
    """Segments [source rank][expert] (the expert-parallel receive layout): segment s multiplies
    expert s % E and starts its own 128-row scale block."""
    from grouped_gemm_opt import _C, quantize_mxfp8
    E, k, n = 4, 256, 576
    seg = [90, 0, 200, 7, 13, 300, 0, 129]
    x, w, _ = gemm_inputs([1] * E, k, n, seed=5)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(sum(seg), k, generator=g).to(torch.bfloat16)
    cnt = torch.tensor(seg)
    xq, xs = quantize_mxfp8(x.to(DEV), cnt.to(DEV))
    wq, ws = quantize_mxfp8(w.to(DEV))
    out = _C.grouped_gemm_mxfp8(xq, xs, wq, ws, cnt.to(DEV), E, True)
    xd = _deq(xq, xs, seg, k)
    wd = _deq(wq, ws, [n] * E, k).view(E, n, k)
    assert_parity(out, oracle.segments_gemm(xd, wd, cnt, E), "mxfp8 segments")


def test_swiglu_mxfp8():
    from grouped_gemm_opt import _C, mxfp8_block_gate_up, quantize_mxfp8
    counts, K, F = [2000, 0, 3000, 77], 256, 200   # F not a multiple of the 128-row block
    E = len(counts)
    x, w, tpe = gemm_inputs(counts, K, 2 * F, seed=2)
    wb = mxfp8_block_gate_up(w.to(DEV))
    assert torch.equal(wb.cpu(), oracle.mx_block_gate_up(w))
    xq, xs = quantize_mxfp8(x.to(DEV), tpe.to(DEV))
    wq, ws = quantize_mxfp8(wb)
    h = _C.grouped_gemm_swiglu_mxfp8(xq, xs, wq, ws, tpe.to(DEV), E, F, True)
    assert h.shape == (x.size(0), F)
    xd = _deq(xq, xs, counts, K)
    rows = wb.size(1)
    wd = oracle.mx_unblock_gate_up(_deq(wq, ws, [rows] * E, K).view(E, rows, K), F)
    assert_parity(h, oracle.swiglu_gemm(xd, wd, tpe, E), "swiglu mxfp8")


def test_fused_moe_mxfp8():
    """MXFP8 layer vs the same quantisation steps on the CPU (dequantised operands, fp32 math)."""
    from grouped_gemm_opt import fused_moe_mxfp8, quantize_moe_weights_mxfp8
    g = torch.Generator().manual_seed(9)
    T, H, F, E, k = 512, 512, 1024, 8, 2
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    wgu = (torch.randn(E, 2 * F, H, generator=g) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(E, H, F, generator=g) * 0.02).to(torch.bfloat16)
    qw = quantize_moe_weights_mxfp8(wgu.to(DEV), wd.to(DEV))
    out = fused_moe_mxfp8(x.to(DEV), logits.to(DEV), qw, k)
    ids, w, tpe = oracle.route(logits.numpy(), k)
    st, pos = oracle.permute_indices(ids, E)
    xs = x[torch.from_numpy(st).long()]
    xq, xsf = oracle.mx_quantize(xs, tpe)
    rows = qw.w_gate_up_q.size(1)
    gud = oracle.mx_unblock_gate_up(_deq(qw.w_gate_up_q, qw.w_gate_up_scale, [rows] * E, H)
                                    .view(E, rows, H), F)
    h = oracle.swiglu_gemm(oracle.mx_dequantize(xq, xsf, tpe, H), gud, torch.from_numpy(tpe), E)
    hq, hsf = oracle.mx_quantize(h.to(torch.bfloat16), tpe)
    dd = _deq(qw.w_down_q, qw.w_down_scale, [H] * E, F).view(E, H, F)
    y = oracle.segments_gemm(oracle.mx_dequantize(hq, hsf, tpe, F), dd, torch.from_numpy(tpe), E)
    ref = oracle.combine(y.to(torch.bfloat16), w, pos)
    assert_parity(out, ref, "fused moe mxfp8")
    rel, cos = parity(out, oracle.moe_layer(x, logits, wgu, wd, k, round_to=torch.bfloat16))
    assert cos > 0.995, cos  # vs the bf16 layer: MX quantisation error only


def test_mxfp8_large_k_many_tiles():
    """32 K stages per tile (the stage ring wraps many times) and a few hundred tiles."""
    from grouped_gemm_opt import grouped_gemm_opt_mxfp8, quantize_mxfp8
    counts, K, N = [512, 640, 384, 512, 0, 1024, 256, 768], 4096, 2048
    x, w, tpe = gemm_inputs(counts, K, N, seed=11)
    xq, xs = quantize_mxfp8(x.to(DEV), tpe.to(DEV))
    wq, ws = quantize_mxfp8(w.to(DEV))
    out = grouped_gemm_opt_mxfp8(xq, xs, wq, ws, tpe.to(DEV))
    xd = _deq(xq, xs, counts, K)
    wd = _deq(wq, ws, [N] * len(counts), K).view(len(counts), N, K)
    assert_parity(out, oracle.sequential_gemm(xd, wd, tpe), "mxfp8 large")



@pytest.mark.parametrize("counts,k", [([3, 0, 250], 384), ([130, 1], 14336), ([40], 128)])
def test_quantize_mxfp8_bit_exact_widths(counts, k):
    """Row widths whose last warp step is partial (K % 256 == 128) and the Mixtral F width."""
    from grouped_gemm_opt import quantize_mxfp8
    g = torch.Generator().manual_seed(k)
    T = sum(counts)
    x = (torch.randn(T, k, generator=g) * torch.logspace(-3, 3, T).unsqueeze(1)).to(torch.bfloat16)
    q, sf = quantize_mxfp8(x.to(DEV), torch.tensor(counts).to(DEV))
    rq, rsf = oracle.mx_quantize(x, counts)
    assert torch.equal(q.cpu().view(torch.uint8), rq)
    assert np.array_equal(sf.cpu().numpy(), rsf)
