"""Fused-MoE stages on the GPU against the CPU oracle: router and permute bit-exact, SwiGLU
gate/up and down GEMMs and the combine within the stated tolerance, and the whole layer."""
import numpy as np
import pytest
import torch

import grouped_gemm_oracle as oracle
from gpu_util import assert_parity
from inputs import gemm_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def C():
    from grouped_gemm_opt import _C
    return _C


def _logits(T, E, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, E, generator=g)


@pytest.mark.parametrize("T,E,k", [(1, 8, 2), (300, 8, 2), (1000, 64, 6), (4096, 256, 8),
                                   (129, 1024, 16), (257, 5, 5)])
def test_route_and_permute_bit_exact(C, T, E, k):
    logits = _logits(T, E, seed=T)
    ids, w, tpe, scratch = C.moe_route(logits.to(DEV), k)
    rid, rw, rtpe = oracle.route(logits.numpy(), k)
    assert np.array_equal(ids.cpu().numpy(), rid)
    assert np.array_equal(tpe.cpu().numpy(), rtpe)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
    H = 64
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    xs, stok, spos = C.moe_permute(x.to(DEV), ids, scratch, E)
    rst, rpos = oracle.permute_indices(rid, E)
    assert np.array_equal(stok.cpu().numpy(), rst)
    assert np.array_equal(spos.cpu().numpy(), rpos)
    assert torch.equal(xs.cpu(), x[torch.from_numpy(rst).long()])


def test_route_ties_lower_index(C):
    logits = torch.zeros(3, 16)
    logits[1, 7] = 1.0
    ids, w, tpe, _ = C.moe_route(logits.to(DEV), 4)
    assert ids.cpu().tolist() == [[0, 1, 2, 3], [7, 0, 1, 2], [0, 1, 2, 3]]


@pytest.mark.parametrize("k", [1, 2, 8])
def test_combine(C, k):
    T, H = 333, 256
    rng = np.random.default_rng(k)
    ids = np.stack([rng.permutation(16)[:k] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    _, pos = oracle.permute_indices(ids, 16)
    y = torch.randn(T * k, H, generator=torch.Generator().manual_seed(k)).to(torch.bfloat16)
    out = C.moe_combine(y.to(DEV), torch.from_numpy(w).to(DEV), torch.from_numpy(pos).to(DEV))
    ref = oracle.combine(y, w, pos)
    # fp32 accumulation then one bf16 rounding: within 1 bf16 ulp of the fp32 oracle
    diff = (out.float().cpu() - ref).abs()
    assert (diff <= ref.abs() * 2.0 ** -8 + 1e-6).all(), diff.max()


@pytest.mark.parametrize("counts,F,K", [([40, 0, 300, 7], 128, 256), ([5, 129, 1], 200, 64),
                                        ([1000, 1000], 1024, 512), ([2000, 0, 3000], 2048, 256)])
def test_swiglu_gemm(C, counts, F, K):
    x, w, tpe = gemm_inputs(counts, K, 2 * F, seed=11)
    ref = oracle.swiglu_gemm(x, w, tpe, len(counts))
    h = C.grouped_gemm_swiglu(x.to(DEV), w.to(DEV), tpe.to(DEV), len(counts), True)
    assert h.shape == (x.size(0), F)
    assert_parity(h, ref, "swiglu")


def test_segments_layout_of_expert_parallel(C):
    """Segments [src rank][local expert], segment s -> expert s % E_local (EP receive layout)."""
    counts = [3, 0, 130, 17, 64, 1]  # 3 sources x 2 local experts
    x, w, _ = gemm_inputs(counts, 128, 192, seed=4)
    w = w[:2].contiguous()
    tpe = torch.tensor(counts)
    ref = oracle.segments_gemm(x, w, tpe, 2)
    for tc in (4, 3):
        out = C.grouped_gemm_segments(x.to(DEV), w.to(DEV), tpe.to(DEV), 2, tc, True)
        assert_parity(out, ref, f"segments tc={tc}")


def _moe_weights(E, H, F, seed):
    g = torch.Generator().manual_seed(seed)
    wgu = (torch.randn(E, 2 * F, H, generator=g) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(E, H, F, generator=g) * 0.02).to(torch.bfloat16)
    return wgu, wd


@pytest.mark.parametrize("T,H,F,E,k", [(512, 256, 512, 8, 2), (256, 1024, 512, 256, 8),
                                       (77, 128, 64, 4, 1)])
def test_fused_moe_small(T, H, F, E, k):
    from grouped_gemm_opt import fused_moe
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    wgu, wd = _moe_weights(E, H, F, seed=E)
    out = fused_moe(x.to(DEV), logits.to(DEV), wgu.to(DEV), wd.to(DEV), k)
    ref = oracle.moe_layer(x, logits, wgu, wd, k, round_to=torch.bfloat16)
    assert_parity(out, ref, "fused_moe")


def test_fused_moe_mixtral_full_size_token_sample():
    """Mixtral layer (T=16384, H=4096, F=14336, E=8, top-2) at full size; every token is
    independent, so a token sample is checked against the oracle run on just those tokens."""
    from grouped_gemm_opt import fused_moe
    T, H, F, E, k = 16384, 4096, 14336, 8, 2
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, device=DEV, generator=g)
    wgu = (torch.randn(E, 2 * F, H, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(E, H, F, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    out = fused_moe(x, logits, wgu, wd, k)
    sel = torch.randperm(T, generator=torch.Generator().manual_seed(0))[:48]
    ref = oracle.moe_layer(x[sel.to(DEV)].cpu(), logits[sel.to(DEV)].cpu(), wgu.cpu(), wd.cpu(),
                           k, round_to=torch.bfloat16)
    assert_parity(out[sel.to(DEV)], ref, "mixtral sample")


@pytest.mark.parametrize("bn", [256, 192, 128])
def test_swiglu_pair_tile_widths(C, bn, monkeypatch):
    monkeypatch.setenv("GGO_PAIR_BN", str(bn))
    # large enough that AUTO picks the CTA-pair kernel; F = 504
    x, w, tpe = gemm_inputs([4000, 0, 6000], 128, 1008, seed=bn)
    ref = oracle.swiglu_gemm(x, w, tpe, 3)
    h = C.grouped_gemm_swiglu(x.to(DEV), w.to(DEV), tpe.to(DEV), 3, True)
    assert_parity(h, ref, f"swiglu pair bn={bn}")


def test_fused_moe_fp16():
    from grouped_gemm_opt import fused_moe
    g = torch.Generator().manual_seed(5)
    T, H, F, E, k = 300, 256, 384, 8, 2
    x = torch.randn(T, H, generator=g).to(torch.float16)
    logits = torch.randn(T, E, generator=g)
    wgu = (torch.randn(E, 2 * F, H, generator=g) * 0.02).to(torch.float16)
    wd = (torch.randn(E, H, F, generator=g) * 0.02).to(torch.float16)
    out = fused_moe(x.to(DEV), logits.to(DEV), wgu.to(DEV), wd.to(DEV), k)
    assert out.dtype == torch.float16
    ref = oracle.moe_layer(x, logits, wgu, wd, k, round_to=torch.float16)
    assert_parity(out, ref, "fused_moe fp16")


@pytest.mark.parametrize("swiglu", [False, True])
def test_scatter_epilogue_single_gpu(C, swiglu):
    """The expert-parallel scatter epilogue with this GPU as the only 'peer': row r of the GEMM
    must land at row origin[r] (& 0x0fffffff) of the target buffer; rows are a random
    permutation, segments [expert-major], capacity larger than the counted rows."""
    counts = [300, 7, 0, 513, 129]
    n_out, k = 256, 512
    x, w, tpe = gemm_inputs(counts, k, 2 * n_out if swiglu else n_out, seed=31)
    rows = x.size(0)
    cap = rows + 100
    xc = torch.zeros(cap, k, dtype=torch.bfloat16)
    xc[:rows] = x
    perm = torch.randperm(rows, generator=torch.Generator().manual_seed(3)).to(torch.int32)
    origin = torch.zeros(cap, dtype=torch.int32)
    origin[:rows] = perm  # source rank 0 in the top bits
    target = torch.zeros(rows, n_out, dtype=torch.bfloat16, device=DEV)
    if swiglu:
        ref = oracle.swiglu_gemm(x, w, tpe, len(counts))
        h = C.ep_grouped_gemm(xc.to(DEV), w.to(DEV), tpe.to(DEV), len(counts), True, None, [],
                              True)
        out = h[:rows]
    else:
        ref = oracle.segments_gemm(x, w, tpe, len(counts))
        C.ep_grouped_gemm(xc.to(DEV), w.to(DEV), tpe.to(DEV), len(counts), False,
                          origin.to(DEV), [target.data_ptr()], True)
        torch.cuda.synchronize()
        out = torch.empty_like(target)
        out[:] = 0
        out = target[perm.long().to(DEV)]
    assert_parity(out, ref, f"scatter swiglu={swiglu}")


@pytest.mark.parametrize("chunks", [1, 4, 7])
def test_fused_moe_host_matches_device_layer(chunks):
    """fused_moe_host (tokens and result in pinned host memory, copies overlapped on side
    streams) gives the device layer's result: every token is computed by the same kernels."""
    from grouped_gemm_opt import StageEvents, fused_moe, fused_moe_host
    g = torch.Generator().manual_seed(9)
    T, H, F, E, k = 1000, 512, 768, 8, 2
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    wgu, wd = _moe_weights(E, H, F, seed=3)
    wgu, wd = wgu.to(DEV), wd.to(DEV)
    timer = StageEvents()
    dev_out = fused_moe(x.to(DEV), logits.to(DEV), wgu, wd, k, timer=timer)
    host_out = fused_moe_host(x.pin_memory(), logits.pin_memory(), wgu, wd, k, chunks=chunks)
    torch.cuda.synchronize()
    assert not host_out.is_cuda and host_out.shape == (T, H)
    assert_parity(host_out, dev_out.cpu(), f"host chunks={chunks}")
    assert_parity(host_out, oracle.moe_layer(x, logits, wgu.cpu(), wd.cpu(), k,
                                             round_to=torch.bfloat16), "host vs oracle")
    ms = timer.ms()
    assert set(ms) == {"route", "dispatch", "gate_up", "down", "combine"}
    assert all(v >= 0 for v in ms.values())


def test_dsv3_decode_layer_token_sample():
    """DeepSeek-V3-shaped layer at decode size (T=256, H=7168, F=2048, E=256, top-8): about 8
    rows per expert, all on skinny tiles; a token sample is checked against the oracle."""
    from grouped_gemm_opt import fused_moe
    T, H, F, E, k = 256, 7168, 2048, 256, 8
    g = torch.Generator(device=DEV).manual_seed(15)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, device=DEV, generator=g)
    wgu = (torch.randn(E, 2 * F, H, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(E, H, F, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    out = fused_moe(x, logits, wgu, wd, k)
    sel = torch.tensor([0, 77, 255])
    ref = oracle.moe_tokens(x[sel.to(DEV)].cpu(), logits[sel.to(DEV)].cpu(),
                            lambda e: (wgu[e].cpu(), wd[e].cpu()), k, round_to=torch.bfloat16)
    assert_parity(out[sel.to(DEV)], ref, "dsv3 decode sample")


def test_host_pipeline_streams_batches():
    """MoEHostPipeline: three batches of different sizes submitted back to back (copies of one
    batch overlapping the layer of another) give each batch's device-layer result."""
    from grouped_gemm_opt import MoEHostPipeline, fused_moe
    g = torch.Generator().manual_seed(13)
    H, F, E, k = 512, 768, 8, 2
    wgu, wd = _moe_weights(E, H, F, seed=5)
    wgu, wd = wgu.to(DEV), wd.to(DEV)
    pipe = MoEHostPipeline(wgu, wd, k)
    batches, outs = [], []
    for T in (700, 1, 1300):
        x = torch.randn(T, H, generator=g).to(torch.bfloat16).pin_memory()
        logits = torch.randn(T, E, generator=g).pin_memory()
        batches.append((x, logits))
        outs.append(pipe.submit(x, logits))
    pipe.synchronize()
    for (x, logits), out in zip(batches, outs):
        assert not out.is_cuda and out.shape == x.shape
        ref = fused_moe(x.to(DEV), logits.to(DEV), wgu, wd, k).cpu()
        assert torch.equal(out, ref), f"pipeline batch of {x.size(0)} tokens differs"
