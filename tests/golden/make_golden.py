"""Generates the golden fixtures in this folder from the REFERENCE implementation itself.

Run in a container where the reference checkout is available (it is not on the GPU box):

    python tests/golden/make_golden.py /path/to/GroupedGEMM-OPT

It imports the reference's ``benchmarks/benchmark.py`` and calls its ground-truth
``sequential_gemm`` (benchmark.py:91-107) and its routing generators ``uniform_distribution`` /
``skewed_distribution`` (benchmark.py:50-69) on CPU tensors. Inputs are regenerated from seeds by
``tests/golden/inputs.py`` (stored here as SHA-256 digests so drift is detected); outputs are
stored as raw bf16 bits (small cases) or as checksums plus a strided sample (cfg1).
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from inputs import EDGE_CASES, cfg1_inputs, edge_inputs  # noqa: E402


def _digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "benchmarks"))
    import benchmark as ref  # the reference's own module

    out = {}
    # cfg1: E=8, T=256, K=512, N=1024, tpe [32]*8, bf16, seed 0
    x, w, tpe = cfg1_inputs()
    y = ref.sequential_gemm(x, w, tpe)
    assert y.dtype == torch.bfloat16 and y.shape == (256, 1024)
    yf = y.double()
    out["cfg1_x_sha"] = np.array(_digest(x))
    out["cfg1_w_sha"] = np.array(_digest(w))
    out["cfg1_row_sum"] = yf.sum(1).numpy()
    out["cfg1_col_sum"] = yf.sum(0).numpy()
    out["cfg1_sample_idx"] = np.arange(0, y.numel(), 61, dtype=np.int64)
    out["cfg1_sample_bits"] = _bits(y.reshape(-1)[torch.from_numpy(out["cfg1_sample_idx"])])

    # edge cases: full outputs at K=128, N=64
    for name, counts in EDGE_CASES.items():
        x, w, tpe = edge_inputs(counts)
        y = ref.sequential_gemm(x, w, tpe)
        out[f"edge_{name}_x_sha"] = np.array(_digest(x))
        out[f"edge_{name}_w_sha"] = np.array(_digest(w))
        out[f"edge_{name}_y_bits"] = _bits(y)

    # routing generators
    for T, E in [(4096, 8), (8192, 64), (1000, 7), (16384, 256)]:
        out[f"uniform_{T}_{E}"] = ref.uniform_distribution(T, E).numpy()
        out[f"skewed_{T}_{E}"] = ref.skewed_distribution(T, E).numpy()

    np.savez_compressed(HERE / "reference_golden.npz", **out)
    print("wrote", HERE / "reference_golden.npz", sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
