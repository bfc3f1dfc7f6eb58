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
