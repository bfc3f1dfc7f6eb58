"""Parity of the tcgen05 grouped GEMM against the CPU oracle (the reference's per-expert
sequential_gemm restated), on seeded inputs. All calls go through the C ABI (via the _C binding
or directly through ctypes)."""
import ctypes

import numpy as np
import pytest
import torch

import grouped_gemm_oracle as oracle
from gpu_util import assert_parity, reference_allclose
from inputs import EDGE_CASES, cfg1_inputs, edge_inputs, gemm_inputs

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def ggo():
    import grouped_gemm_opt
    return grouped_gemm_opt


def test_cfg1_all_tile_configs(ggo):
    x, w, tpe = cfg1_inputs()
    ref = oracle.sequential_gemm(x, w, tpe)
    xd, wd = x.to(DEV), w.to(DEV)
    for tc in ggo.TileConfig:
        for sort in (False, True):
            out = ggo.grouped_gemm_opt(xd, wd, tpe, tc, sort_by_m=sort)
            torch.cuda.synchronize()
            assert out.shape == (256, 1024) and out.dtype == torch.bfloat16
            assert_parity(out, ref, f"cfg1 tc={tc.name} sort={sort}")
            assert reference_allclose(out, ref)


def test_cfg1_gpu_counts_no_host_copy(ggo):
    x, w, tpe = cfg1_inputs()
    ref = oracle.sequential_gemm(x, w, tpe)
    out = ggo.grouped_gemm_opt(x.to(DEV), w.to(DEV), tpe.to(DEV))
    assert_parity(out, ref, "cfg1 gpu counts")
    ggo.check_device_errors(0)


@pytest.mark.parametrize("name", list(EDGE_CASES))
@pytest.mark.parametrize("tc", [0, 1, 3, 4])
def test_edge_cases(ggo, name, tc):
    x, w, tpe = edge_inputs(EDGE_CASES[name])
    ref = oracle.sequential_gemm(x, w, tpe)
    out = ggo.grouped_gemm_opt(x.to(DEV), w.to(DEV), tpe.to(DEV), tc)
    assert_parity(out, ref, f"{name} tc={tc}")
    ggo.check_device_errors(0)


@pytest.mark.parametrize("k,n", [(200, 1000), (8, 8), (4096, 136), (72, 520)])
def test_odd_k_and_n(ggo, k, n):
    x, w, tpe = gemm_inputs([3, 0, 130, 61, 1], k, n, seed=3)
    ref = oracle.sequential_gemm(x, w, tpe)
    for tc in (0, 1, 3):
        out = ggo.grouped_gemm_opt(x.to(DEV), w.to(DEV), tpe, tc)
        assert_parity(out, ref, f"k={k} n={n} tc={tc}")


def test_fp16(ggo):
    x, w, tpe = gemm_inputs([17, 300, 0, 64], 256, 384, seed=5, dtype=torch.float16)
    ref = oracle.sequential_gemm(x, w, tpe)
    for tc in (0, 1, 3):
        out = ggo.grouped_gemm_opt(x.to(DEV), w.to(DEV), tpe.to(DEV), tc)
        assert out.dtype == torch.float16
        assert_parity(out, ref, f"fp16 tc={tc}")
        assert reference_allclose(out, ref, torch.float16)


def test_many_experts_zero_counts(ggo):
    tpe = oracle.dirichlet_counts(2048, 256, seed=1)
    assert (tpe == 0).any()
    x, w, _ = gemm_inputs(tpe, 256, 256, seed=7)
    ref = oracle.sequential_gemm(x, w, tpe)
    for sort in (False, True):
        for tc in (4, 3):
            out = ggo.grouped_gemm_opt(x.to(DEV), w.to(DEV), tpe.to(DEV), tc, sort_by_m=sort)
            assert_parity(out, ref, f"E=256 sort={sort} tc={tc}")


def test_empty_input(ggo):
    w = torch.randn(4, 64, 32, device=DEV, dtype=torch.bfloat16)
    out = ggo.grouped_gemm_opt(torch.empty(0, 32, device=DEV, dtype=torch.bfloat16), w,
                               torch.zeros(4, dtype=torch.int64))
    assert out.shape == (0, 64)


def test_count_mismatch(ggo):
    x = torch.randn(10, 32, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(2, 64, 32, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        ggo.grouped_gemm_opt(x, w, torch.tensor([3, 4]))
    ggo.grouped_gemm_opt(x, w, torch.tensor([3, 4], device=DEV))
    with pytest.raises(RuntimeError):
        ggo.check_device_errors(0)
    ggo.check_device_errors(0)  # cleared


def test_bad_arguments(ggo):
    x = torch.randn(10, 30, device=DEV, dtype=torch.bfloat16)  # K not a multiple of 8
    w = torch.randn(2, 64, 30, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        ggo.grouped_gemm_opt(x, w, torch.tensor([5, 5]))
    with pytest.raises(RuntimeError):
        ggo.grouped_gemm_opt(torch.randn(4, 32, device=DEV, dtype=torch.float32),
                             torch.randn(1, 8, 32, device=DEV, dtype=torch.float32),
                             torch.tensor([4]))
    with pytest.raises(RuntimeError):  # K mismatch
        ggo.grouped_gemm_opt(torch.randn(4, 32, device=DEV, dtype=torch.bfloat16),
                             torch.randn(1, 8, 64, device=DEV, dtype=torch.bfloat16),
                             torch.tensor([4]))


def test_triton_aliases(ggo):
    x, w, tpe = edge_inputs(EDGE_CASES["span_gt4"])
    ref = oracle.sequential_gemm(x, w, tpe)
    assert_parity(ggo.triton_fused_moe(x.to(DEV), w.to(DEV), tpe), ref, "triton_fused_moe")
    assert_parity(ggo.triton_grouped_gemm(x.to(DEV), w.to(DEV), tpe, BLOCK_N=256), ref,
                  "triton_grouped_gemm")


def _sample_rows(tpe, per_expert=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    rows, off = [], 0
    for m in tpe.tolist():
        if m > 0:
            rows.append(off + torch.randint(0, m, (min(per_expert, m),), generator=g))
        off += m
    return torch.cat(rows)


def _ref_rows(x, w, tpe, rows):
    """CPU fp32 reference for the sampled rows, one weight copy per expert touched."""
    ex = torch.searchsorted(torch.cumsum(tpe, 0), rows, right=True)
    xs = x[rows.to(x.device)].float().cpu()
    ref = torch.empty(rows.numel(), w.size(1))
    for e in ex.unique().tolist():
        sel = (ex == e).nonzero().flatten()
        ref[sel] = xs[sel] @ w[e].float().cpu().T
    return ref


@pytest.mark.parametrize("tc", [4, 1])
@pytest.mark.parametrize("dist", ["uniform", "readme", "skewed"])
def test_cfg2_full_size_sampled_rows(ggo, dist, tc):
    """cfg2 (E=8, T=4096, K=4096, N=14336) at full size; a row sample is checked on the CPU."""
    T, E, K, N = 4096, 8, 4096, 14336
    tpe = {"uniform": oracle.uniform_distribution(T, E),
           "readme": torch.tensor([512, 480, 520, 500, 510, 490, 530, 554]),
           "skewed": oracle.skewed_distribution(T, E)}[dist]
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(T, K, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(E, N, K, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    out = ggo.grouped_gemm_opt(x, w, tpe.to(DEV), tc)
    rows = _sample_rows(tpe)
    ref = _ref_rows(x, w, tpe, rows)
    assert_parity(out[rows.to(DEV)], ref, f"cfg2 {dist} tc={tc}")
    ggo.check_device_errors(0)


def test_cfg3_skewed_many_experts_sampled_rows(ggo):
    T, E, K, N = 8192, 64, 4096, 14336
    for tpe in (oracle.zipf_counts(T, E, seed=0), oracle.dirichlet_counts(T, E, seed=0)):
        g = torch.Generator(device=DEV).manual_seed(1)
        x = torch.randn(T, K, device=DEV, generator=g).to(torch.bfloat16)
        w = (torch.randn(E, N, K, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
        out = ggo.grouped_gemm_opt(x, w, tpe.to(DEV))
        rows = _sample_rows(tpe, 4)
        ref = _ref_rows(x, w, tpe, rows)
        assert_parity(out[rows.to(DEV)], ref, "cfg3")
        del w
        torch.cuda.empty_cache()


def test_c_abi_direct_ctypes():
    """Calls ggo_grouped_gemm through ctypes with raw device pointers: no torch in the ABI."""
    import grouped_gemm_opt  # noqa: F401  (initialises the CUDA context through torch)
    from build_ext import lib_path
    lib = ctypes.CDLL(str(lib_path()))
    x, w, tpe = edge_inputs(EDGE_CASES["ragged"])
    ref = oracle.sequential_gemm(x, w, tpe)
    xd, wd, td = x.to(DEV), w.to(DEV), tpe.to(DEV)
    out = torch.empty(x.size(0), w.size(1), device=DEV, dtype=torch.bfloat16)
    lib.ggo_workspace_size.restype = ctypes.c_size_t
    ws = torch.zeros(lib.ggo_workspace_size(), dtype=torch.uint8, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    f = lib.ggo_grouped_gemm
    f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                          ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_void_p, ctypes.c_void_p]
    for _ in range(2):
        st = f(xd.data_ptr(), wd.data_ptr(), out.data_ptr(), td.data_ptr(), w.size(0), x.size(0),
               w.size(1), w.size(2), 0, 4, 1, ws.data_ptr(), stream)
        assert st == 0
        torch.cuda.synchronize()
        assert_parity(out, ref, "ctypes")
    code = ctypes.c_int(-1)
    lib.ggo_workspace_error.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    assert lib.ggo_workspace_error(ws.data_ptr(), stream, ctypes.byref(code)) == 0
    assert code.value == 0
    # the counters are back at zero after each launch
    assert ws[:8].sum().item() == 0


@pytest.mark.parametrize("bn", [256, 224, 192, 160, 128])
def test_pair_tile_widths(ggo, bn, monkeypatch):
    """Every CTA-pair tile width, forced through GGO_PAIR_BN (plain epilogue)."""
    monkeypatch.setenv("GGO_PAIR_BN", str(bn))
    x, w, tpe = gemm_inputs([300, 0, 17, 513, 256], 192, 1000, seed=bn)
    ref = oracle.sequential_gemm(x, w, tpe)
    out = ggo.grouped_gemm_opt(x.to(DEV), w.to(DEV), tpe.to(DEV), 3)
    assert_parity(out, ref, f"pair bn={bn}")


@pytest.mark.parametrize("gm", [1, 3, 8, 16])
def test_raster_group_sizes(ggo, gm, monkeypatch):
    monkeypatch.setenv("GGO_RASTER_GROUP_M", str(gm))
    x, w, tpe = gemm_inputs([1100, 5, 700], 128, 640, seed=gm)
    ref = oracle.sequential_gemm(x, w, tpe)
    for tc in (1, 3):
        out = ggo.grouped_gemm_opt(x.to(DEV), w.to(DEV), tpe.to(DEV), tc)
        assert_parity(out, ref, f"group_m={gm} tc={tc}")


@pytest.mark.parametrize("chunks", [1, 3, 8])
def test_host_buffer_api(ggo, chunks):
    """grouped_gemm_opt_host: pinned host activations/output, overlapped per expert chunk."""
    x, w, tpe = gemm_inputs([300, 0, 17, 513, 256, 0, 90, 1], 256, 384, seed=chunks)
    ref = oracle.sequential_gemm(x, w, tpe)
    out = ggo.grouped_gemm_opt_host(x.pin_memory(), w.to(DEV), tpe, chunks=chunks)
    torch.cuda.synchronize()
    assert not out.is_cuda
    assert_parity(out, ref, f"host api chunks={chunks}")


@pytest.mark.parametrize("tc", [0, 1, 3, 4])
@pytest.mark.parametrize("counts,n,k", [([300, 0, 17, 513, 256], 256, 384),
                                        ([1, 7, 8, 127, 128, 129], 200, 1000),
                                        ([4000, 3000], 512, 2048)])
def test_dgrad(tc, counts, n, k):
    """dx = dy @ W[e] per segment (weights read MN-major in place)."""
    from grouped_gemm_opt import _C
    g = torch.Generator().manual_seed(len(counts) + tc)
    tpe = torch.tensor(counts)
    dy = torch.randn(int(tpe.sum()), n, generator=g).to(torch.bfloat16)
    w = (torch.randn(len(counts), n, k, generator=g) * 0.05).to(torch.bfloat16)
    wt = w.transpose(1, 2).contiguous()  # [E, K, N]: dgrad is a forward GEMM with W^T
    ref = oracle.sequential_gemm(dy, wt, tpe)
    dx = _C.grouped_gemm_dgrad(dy.to(DEV), w.to(DEV), tpe.to(DEV), tc, True)
    assert dx.shape == (dy.size(0), k)
    assert_parity(dx, ref, f"dgrad tc={tc} n={n} k={k}")


def _wgrad_ref(x, dy, tpe):
    outs, off = [], 0
    for m in tpe.tolist():
        outs.append(dy[off:off + m].float().T @ x[off:off + m].float())
        off += m
    return torch.stack(outs)


@pytest.mark.parametrize("sort", [False, True])
@pytest.mark.parametrize("counts,n,k", [([300, 0, 17, 513, 256], 256, 384),
                                        ([1, 7, 63, 64, 65, 130, 0], 200, 1000),
                                        ([4000, 3000], 512, 2048),
                                        ([0, 0, 5], 64, 64)])
@pytest.mark.parametrize("pair", ["0", "2"])
def test_wgrad(sort, counts, n, k, pair, monkeypatch):
    """dw[e] = dy_e^T @ x_e over each expert's own tokens (zero for experts without tokens), on
    the single-CTA kernel and on the CTA-pair kernel (forced; AUTO pairs only large problems)."""
    from grouped_gemm_opt import _C
    monkeypatch.setenv("GGO_WGRAD_PAIR", pair)
    g = torch.Generator().manual_seed(len(counts) * 7 + k)
    tpe = torch.tensor(counts)
    T = int(tpe.sum())
    x = torch.randn(T, k, generator=g).to(torch.bfloat16)
    dy = torch.randn(T, n, generator=g).to(torch.bfloat16)
    ref = _wgrad_ref(x, dy, tpe)
    dw = _C.grouped_gemm_wgrad(x.to(DEV), dy.to(DEV), tpe.to(DEV), sort)
    assert dw.shape == (len(counts), n, k)
    for e, m in enumerate(counts):
        if m == 0:
            assert (dw[e] == 0).all()
        else:
            assert_parity(dw[e], ref[e], f"wgrad expert {e} (m={m})")


def test_autograd_matches_torch_reference(ggo):
    """Backward through grouped_gemm_opt vs autograd of the per-expert F.linear loop (fp32)."""
    x, w, tpe = gemm_inputs([130, 0, 64, 257, 9], 256, 320, seed=21)
    go = torch.randn(x.size(0), 320, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    xr = x.float().requires_grad_()
    wr = w.float().requires_grad_()
    yr = oracle.sequential_gemm(xr, wr, tpe)
    yr.backward(go.float())
    xd = x.to(DEV).requires_grad_()
    wd = w.to(DEV).requires_grad_()
    y = ggo.grouped_gemm_opt(xd, wd, tpe.to(DEV))
    y.backward(go.to(DEV))
    assert_parity(y, yr, "forward")
    assert_parity(xd.grad, xr.grad, "grad input")
    for e in range(w.size(0)):
        if int(tpe[e]) == 0:
            assert (wd.grad[e] == 0).all()
        else:
            assert_parity(wd.grad[e], wr.grad[e], f"grad weight {e}")


@pytest.mark.parametrize("split", ["0", "1"])
def test_split_tail_launch(ggo, split, monkeypatch):
    """Pair pass + single-CTA pass over short segment tails (count mod 256 in 1..128)."""
    monkeypatch.setenv("GGO_SPLIT_TAILS", split)
    monkeypatch.setenv("GGO_SPLIT_MIN_TILES", "1")  # split even this small problem
    counts = [256 * 3 + 5, 128, 129, 0, 256, 383, 384, 1, 600]
    x, w, tpe = gemm_inputs(counts, 256, 512, seed=9)
    ref = oracle.sequential_gemm(x, w, tpe)
    out = ggo.grouped_gemm_opt(x.to(DEV), w.to(DEV), tpe.to(DEV), 3)
    assert_parity(out, ref, f"split={split}")


@pytest.mark.parametrize("tc", [1, 3])
def test_dgrad_wgrad_fp16(tc, monkeypatch):
    from grouped_gemm_opt import _C
    monkeypatch.setenv("GGO_WGRAD_PAIR", "2" if tc == 3 else "0")
    g = torch.Generator().manual_seed(tc)
    counts = [700, 0, 300, 1100, 20]
    tpe = torch.tensor(counts)
    T, n, k = int(tpe.sum()), 256, 512
    dy = torch.randn(T, n, generator=g).to(torch.float16)
    x = torch.randn(T, k, generator=g).to(torch.float16)
    w = (torch.randn(len(counts), n, k, generator=g) * 0.05).to(torch.float16)
    dx = _C.grouped_gemm_dgrad(dy.to(DEV), w.to(DEV), tpe.to(DEV), tc, True)
    assert dx.dtype == torch.float16
    assert_parity(dx, oracle.sequential_gemm(dy, w.transpose(1, 2).contiguous(), tpe), "dgrad fp16")
    dw = _C.grouped_gemm_wgrad(x.to(DEV), dy.to(DEV), tpe.to(DEV), True)
    ref = _wgrad_ref(x, dy, tpe)
    for e, m in enumerate(counts):
        if m:
            assert_parity(dw[e], ref[e], f"wgrad fp16 {e}")


def test_backward_cfg2_full_size_sampled():
    """dgrad and wgrad at the cfg2 shapes (E=8, T=4096, K=4096, N=14336), checked on samples:
    dx rows (each row is independent) and dW columns of one expert."""
    from grouped_gemm_opt import _C
    T, E, K, N = 4096, 8, 4096, 14336
    tpe = torch.tensor([512, 480, 520, 500, 510, 490, 530, 554])
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(T, K, device=DEV, generator=g).to(torch.bfloat16)
    dy = torch.randn(T, N, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(E, N, K, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    dx = _C.grouped_gemm_dgrad(dy, w, tpe.to(DEV), 4, True)
    rows = _sample_rows(tpe, 4)
    ex = torch.searchsorted(torch.cumsum(tpe, 0), rows, right=True)
    ref = torch.stack([dy[int(r)].float().cpu() @ w[int(e)].float().cpu()
                       for r, e in zip(rows, ex)])
    assert_parity(dx[rows.to(DEV)], ref, "dgrad cfg2")
    dw = _C.grouped_gemm_wgrad(x, dy, tpe.to(DEV), True)
    e = 7
    off = int(tpe[:e].sum())
    cols = torch.randint(0, K, (16,), generator=torch.Generator().manual_seed(1))
    ref = dy[off:off + 554].float().cpu().T @ x[off:off + 554][:, cols.to(DEV)].float().cpu()
    assert_parity(dw[e][:, cols.to(DEV)], ref, "wgrad cfg2 expert 7")


SKINNY_COUNTS = [1, 7, 8, 63, 64, 65, 16, 17, 0, 31, 32, 33, 128 + 5, 256 + 64]


@pytest.mark.parametrize("tc", [0, 1, 4])
@pytest.mark.parametrize("skinny", ["64", "0"])
def test_skinny_segments(ggo, tc, skinny, monkeypatch):
    """Short segments (and short last blocks of longer ones) run swapped-operand tiles: weight
    rows on the MMA's M side, the segment's rows on its N side. Both that path and the 128-row
    path (GGO_SKINNY_ROWS=0) must match the oracle, N not a multiple of the tile width."""
    monkeypatch.setenv("GGO_SKINNY_ROWS", skinny)
    x, w, tpe = gemm_inputs(SKINNY_COUNTS, 320, 640, seed=11)
    ref = oracle.sequential_gemm(x, w, tpe)
    out = ggo.grouped_gemm_opt(x.to(DEV), w.to(DEV), tpe.to(DEV), tc)
    assert_parity(out, ref, f"skinny={skinny} tc={tc}")
    ggo.check_device_errors(0)


@pytest.mark.parametrize("skinny", ["64", "0"])
def test_skinny_swiglu_and_fp16(ggo, skinny, monkeypatch):
    from grouped_gemm_opt import _C
    monkeypatch.setenv("GGO_SKINNY_ROWS", skinny)
    x, w, tpe = gemm_inputs(SKINNY_COUNTS, 256, 2 * 384, seed=12)
    ref = oracle.swiglu_gemm(x, w, tpe, len(SKINNY_COUNTS))
    h = _C.grouped_gemm_swiglu(x.to(DEV), w.to(DEV), tpe.to(DEV), len(SKINNY_COUNTS), True)
    assert_parity(h, ref, f"skinny swiglu={skinny}")
    x, w, tpe = gemm_inputs(SKINNY_COUNTS, 192, 520, seed=13, dtype=torch.float16)
    out = ggo.grouped_gemm_opt(x.to(DEV), w.to(DEV), tpe.to(DEV))
    assert out.dtype == torch.float16
    assert_parity(out, oracle.sequential_gemm(x, w, tpe), f"skinny fp16={skinny}")


def test_skinny_decode_shape(ggo):
    """DSv3-decode-like grouped GEMM: 256 experts of about 8 rows, K=7168, N=4096."""
    g = torch.Generator().manual_seed(14)
    tpe = torch.bincount(torch.randint(0, 256, (2048,), generator=g), minlength=256)
    x = torch.randn(2048, 7168, generator=g).to(torch.bfloat16)
    wd = (torch.randn(256, 4096, 7168, device=DEV) * 0.02).to(torch.bfloat16)
    out = ggo.grouped_gemm_opt(x.to(DEV), wd, tpe.to(DEV))
    # check the rows of a few experts (each row depends only on its expert's weights)
    off = torch.cat([torch.zeros(1, dtype=torch.int64), tpe.cumsum(0)])
    for e in (0, 17, 100, 255):
        a, b = int(off[e]), int(off[e + 1])
        ref = torch.nn.functional.linear(x[a:b].float(), wd[e].float().cpu())
        assert_parity(out[a:b], ref, f"decode expert {e}")
