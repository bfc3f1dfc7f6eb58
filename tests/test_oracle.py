"""Pins the CPU oracle against golden vectors produced by the reference's own benchmark.py
(tests/golden/make_golden.py): its ground-truth ``sequential_gemm`` and routing generators."""
import hashlib
import os

import numpy as np
import pytest
import torch

import grouped_gemm_oracle as oracle
from inputs import EDGE_CASES, cfg1_inputs, edge_inputs

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_golden.npz"))


def _sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _from_bits(bits):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).float()


def test_seeded_inputs_reproduce():
    x, w, _ = cfg1_inputs()
    assert _sha(x) == str(GOLDEN["cfg1_x_sha"])
    assert _sha(w) == str(GOLDEN["cfg1_w_sha"])


def _close_to_bf16_reference(mine_fp32, ref_bf16):
    # The reference output is the bf16 rounding of (nearly) the same fp32 products: at most one
    # bf16 ulp (2^-8 relative) apart, plus a small absolute floor for near-zero outputs.
    diff = (mine_fp32 - ref_bf16).abs()
    tol = ref_bf16.abs() * 2.0 ** -7 + 2e-3
    return bool((diff <= tol).all()), float(diff.max())


def test_sequential_gemm_cfg1_matches_reference():
    x, w, tpe = cfg1_inputs()
    y = oracle.sequential_gemm(x, w, tpe)
    # Sums of the bf16-rounded oracle vs sums of the reference's bf16 output: the two differ only
    # where one rounding lands on the neighbouring bf16 value (<= 1 ulp ~ 2^-8 * |y|, |y| < 2.2).
    yb = y.to(torch.bfloat16).double()
    np.testing.assert_allclose(yb.sum(1).numpy(), GOLDEN["cfg1_row_sum"], atol=0.02)
    np.testing.assert_allclose(yb.sum(0).numpy(), GOLDEN["cfg1_col_sum"], atol=0.02)
    idx = torch.from_numpy(GOLDEN["cfg1_sample_idx"])
    ok, mx = _close_to_bf16_reference(y.reshape(-1)[idx], _from_bits(GOLDEN["cfg1_sample_bits"]))
    assert ok, mx


@pytest.mark.parametrize("name", list(EDGE_CASES))
def test_sequential_gemm_edge_cases_match_reference(name):
    x, w, tpe = edge_inputs(EDGE_CASES[name])
    assert _sha(x) == str(GOLDEN[f"edge_{name}_x_sha"])
    assert _sha(w) == str(GOLDEN[f"edge_{name}_w_sha"])
    y = oracle.sequential_gemm(x, w, tpe)
    ref = _from_bits(GOLDEN[f"edge_{name}_y_bits"]).view(y.shape)
    ok, mx = _close_to_bf16_reference(y, ref)
    assert ok, mx


def test_segments_form_equals_sequential():
    x, w, tpe = edge_inputs(EDGE_CASES["zero_ends"])
    a = oracle.sequential_gemm(x, w, tpe)
    b = oracle.segments_gemm(x, w, tpe, w.size(0))
    assert torch.equal(a, b)


@pytest.mark.parametrize("T,E", [(4096, 8), (8192, 64), (1000, 7), (16384, 256)])
def test_distributions_bit_exact(T, E):
    assert np.array_equal(oracle.uniform_distribution(T, E).numpy(), GOLDEN[f"uniform_{T}_{E}"])
    assert np.array_equal(oracle.skewed_distribution(T, E).numpy(), GOLDEN[f"skewed_{T}_{E}"])


def test_cfg3_generators_are_seeded_and_sum():
    a = oracle.zipf_counts(8192, 64, seed=0)
    b = oracle.zipf_counts(8192, 64, seed=0)
    assert torch.equal(a, b) and int(a.sum()) == 8192 and a[0] > a[-1]
    d = oracle.dirichlet_counts(8192, 64, seed=0)
    assert int(d.sum()) == 8192 and int((d == 0).sum()) > 0


def test_route_permute_properties():
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((300, 16)).astype(np.float32)
    ids, w, tpe = oracle.route(logits, 4)
    assert ids.shape == (300, 4) and np.allclose(w.sum(1), 1, atol=1e-6)
    assert all(len(set(r)) == 4 for r in ids.tolist())
    # descending logits per row
    vals = np.take_along_axis(logits, ids.astype(np.int64), 1)
    assert (np.diff(vals, axis=1) <= 0).all()
    st, pos = oracle.permute_indices(ids, 16)
    assert sorted(pos.tolist()) == list(range(1200))
    flat = ids.reshape(-1)
    # sorted rows are expert-major, token-ascending inside an expert
    e_sorted = flat[np.argsort(pos)]
    assert (np.diff(e_sorted) >= 0).all()
    assert np.array_equal(np.bincount(flat, minlength=16), tpe)
    for e in range(16):
        toks = st[e_sorted == e]
        assert (np.diff(toks) > 0).all()


def test_route_tie_break_lower_index():
    logits = np.zeros((2, 6), dtype=np.float32)
    ids, w, _ = oracle.route(logits, 3)
    assert ids.tolist() == [[0, 1, 2], [0, 1, 2]]
    assert np.allclose(w, 1 / 3)


@pytest.mark.parametrize("name", list(EDGE_CASES))
def test_oracle_matches_reference_triton_grouped_gemm(name):
    """The reference's own triton_grouped_gemm (run in Triton's CPU interpreter, fp32) agrees with
    the oracle: a second, independent pin of the grouped-GEMM semantics."""
    x, w, tpe = edge_inputs(EDGE_CASES[name])
    y = oracle.sequential_gemm(x, w, tpe).double()
    np.testing.assert_allclose(y.sum(1).numpy(), GOLDEN[f"tgg_{name}_row_sum"], atol=1e-3)
    np.testing.assert_allclose(y.sum(0).numpy(), GOLDEN[f"tgg_{name}_col_sum"], atol=1e-3)
    np.testing.assert_allclose(y.reshape(-1)[::37].numpy(), GOLDEN[f"tgg_{name}_sample"],
                               rtol=1e-5, atol=1e-5)


def test_reference_triton_fused_moe_bug_is_not_reproduced():
    """The reference's triton_fused_moe handles at most 4 experts per 128-row tile
    (triton_fused_moe.py:54-73, 131); on a tile spanning more it computes wrong rows. The fixture
    holds its output: it differs from the oracle there (and only there), while this library's
    triton_fused_moe follows the oracle (GPU test test_triton_aliases)."""
    for name in EDGE_CASES:
        x, w, tpe = edge_inputs(EDGE_CASES[name])
        y = oracle.sequential_gemm(x, w, tpe).double()
        dev = np.abs(y.reshape(-1)[::37].numpy() - GOLDEN[f"tfm_{name}_sample"]).max()
        if name == "span_gt4":
            assert dev > 0.1, dev
        else:
            assert dev < 1e-4, (name, dev)


# ----------------------------------------------------------------------------- MXFP8 oracle
def test_mx_scale_exponent_known_answers():
    """X = floor(log2 amax) - 8, +1 above 1.75 * 2^floor, clamped; zero groups -127."""
    amax = np.array([448, 449, 1, 0, 1.75, 1.7500001, 2.0 ** -130, 3e38, 2.0 ** -119],
                    dtype=np.float32)
    assert oracle.mx_scale_exponent(amax).tolist() == [0, 1, -8, -127, -8, -7, -127, 120, -127]


def test_mx_quantize_known_answers():
    x = torch.zeros(130, 128)
    x[0, :3] = torch.tensor([448.0, 1.0, -0.5])    # group 0 of row 0: X = 0, exact
    x[129, 64:67] = torch.tensor([450.0, 226.0, 232.0])  # group 2 of row 129: X = 1
    q, sf = oracle.mx_quantize(x.to(torch.bfloat16), [130])
    assert q[0, :3].tolist() == [0x7E, 0x38, 0xB0]  # e4m3 bits of 448, 1, -0.5
    # 225 -> 224, 113 -> 112, and the tie 116 -> 112 (nearest even)
    assert q[129, 64:67].tolist() == [0x76, 0x6E, 0x6E]
    assert sf.size == (2 + 1) * 1 * 512
    assert sf[0] == 127 and sf[(1 * 1 + 0) * 512 + 1 * 16 + 0 * 4 + 2] == 128
    assert sf[1] == 0  # an all-zero group: X = -127
    # padding rows of the second block keep zero bytes
    assert sf[512 + 2 * 16] == 0


def test_mx_round_trip_error_bound():
    """|dequant(quant(x)) - x| <= max(|x| / 16, half an e4m3 subnormal step) per element."""
    g = torch.Generator().manual_seed(3)
    counts = [100, 0, 150, 50]
    x = (torch.randn(300, 256, generator=g) * torch.logspace(-3, 3, 300).unsqueeze(1)).to(
        torch.bfloat16)
    q, sf = oracle.mx_quantize(x, counts)
    d = oracle.mx_dequantize(q, sf, counts, 256)
    xf = x.float()
    xe = oracle.mx_scale_exponent(xf.view(300, 8, 32).abs().amax(-1).numpy())
    step = torch.from_numpy(np.ldexp(1.0, xe - 10).astype(np.float32)).repeat_interleave(32, 1)
    assert bool(((d - xf).abs() <= torch.maximum(xf.abs() / 16, step)).all())


def test_mx_gate_up_blocking_round_trip():
    w = torch.randn(3, 2 * 200, 128)
    b = oracle.mx_block_gate_up(w)
    assert b.shape == (3, 2 * 256, 128)
    # block 0: gate rows 0..127 then up rows 0..127
    assert torch.equal(b[:, :128], w[:, :128]) and torch.equal(b[:, 128:256], w[:, 200:328])
    assert torch.equal(oracle.mx_unblock_gate_up(b, 200), w)


def test_moe_tokens_equals_layer_rows():
    """The sample form of the layer oracle (used by the expert-parallel parity checks) gives the
    same rows as the whole-layer oracle, and the native-dtype form stays within bf16 rounding."""
    g = torch.Generator().manual_seed(4)
    T, H, F, E, k = 96, 64, 48, 8, 3
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    wgu = (torch.randn(E, 2 * F, H, generator=g) * 0.1).to(torch.bfloat16)
    wd = (torch.randn(E, H, F, generator=g) * 0.1).to(torch.bfloat16)
    full = oracle.moe_layer(x, logits, wgu, wd, k, round_to=torch.bfloat16)
    idx = torch.tensor([0, 5, 17, 40, 41, 95])
    part = oracle.moe_tokens(x[idx], logits[idx], lambda e: (wgu[e], wd[e]), k,
                             round_to=torch.bfloat16)
    assert torch.allclose(part, full[idx], rtol=1e-5, atol=1e-6)
    nat = oracle.moe_layer(x, logits, wgu, wd, k, native=True)
    rel = ((nat - full).abs().max() / full.abs().max()).item()
    assert rel < 2e-2, rel
