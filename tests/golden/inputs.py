"""Seeded input generators shared by the golden-fixture script and the tests.

All tensors are generated on the CPU with ``torch.Generator`` so the same values appear on every
machine with this torch build (the fixtures store SHA-256 digests to detect drift).
"""
from __future__ import annotations

import torch

# Edge cases (counts per expert). Each exercises a case the reference's kernels handle specially
# or get wrong: zero-token experts at the ends, M around the 128-row tile, a tile spanning more
# than four experts (wrong in the reference's triton_fused_moe.py:54-73), one hot expert.
EDGE_CASES = {
    "ragged": [1, 7, 8, 127, 128, 129, 255, 256, 257],
    "zero_ends": [0, 40, 0, 200, 3, 0],
    "span_gt4": [100, 1, 1, 1, 1, 1, 1, 0, 2, 0, 148],
    "one_hot": [0, 0, 300, 0],
    "single": [5],
}
EDGE_K = 128
EDGE_N = 64


def cfg1_inputs(seed: int = 0):
    """x [256,512] ~N(0,1), W [8,1024,512] ~N(0,0.02), tpe [32]*8, bf16."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(256, 512, generator=g).to(torch.bfloat16)
    w = (torch.randn(8, 1024, 512, generator=g) * 0.02).to(torch.bfloat16)
    tpe = torch.full((8,), 32, dtype=torch.int64)
    return x, w, tpe


def edge_inputs(counts, seed: int = 1, k: int = EDGE_K, n: int = EDGE_N):
    g = torch.Generator().manual_seed(seed)
    tpe = torch.tensor(counts, dtype=torch.int64)
    x = torch.randn(int(tpe.sum()), k, generator=g).to(torch.bfloat16)
    w = (torch.randn(len(counts), n, k, generator=g) * 0.05).to(torch.bfloat16)
    return x, w, tpe


def gemm_inputs(counts, k: int, n: int, seed: int = 0, dtype=torch.bfloat16, w_std: float = 0.02):
    """Generic seeded case: x ~N(0,1) [sum(counts), k], W ~N(0,w_std) [E, n, k]."""
    g = torch.Generator().manual_seed(seed)
    tpe = torch.as_tensor(counts, dtype=torch.int64)
    x = torch.randn(int(tpe.sum()), k, generator=g).to(dtype)
    w = (torch.randn(tpe.numel(), n, k, generator=g) * w_std).to(dtype)
    return x, w, tpe
