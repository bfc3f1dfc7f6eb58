"""Generates the golden fixtures in this folder from the REFERENCE implementation itself.

Run in a container where the reference checkout is available (it is not on the GPU box):

    python tests/golden/make_golden.py /path/to/GroupedGEMM-OPT

It imports the reference's ``benchmarks/benchmark.py`` and calls its ground-truth
``sequential_gemm`` (benchmark.py:91-107) and its routing generators ``uniform_distribution`` /
``skewed_distribution`` (benchmark.py:50-69) on CPU tensors. It also runs the reference's own
Triton kernels ``triton_grouped_gemm`` (grouped_gemm_opt/triton_grouped_gemm.py:139-197) and
``triton_fused_moe`` (grouped_gemm_opt/triton_fused_moe.py:104-150) on the CPU under Triton's
interpreter (TRITON_INTERPRET=1, fp32 inputs; the interpreter does not support bf16 here) and
stores checksums of their outputs. Inputs are regenerated from seeds by
``tests/golden/inputs.py`` (stored here as SHA-256 digests so drift is detected); outputs are
stored as raw bf16 bits (small cases) or as checksums plus a strided sample (cfg1).
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
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

    # the reference's Triton kernels under the interpreter (fp32), on the edge cases
    os.environ["TRITON_INTERPRET"] = "1"

    def load(name, rel):
        spec = importlib.util.spec_from_file_location(name, str(Path(ref_root) / rel))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod

    tgg = load("ref_triton_grouped_gemm", "grouped_gemm_opt/triton_grouped_gemm.py")
    tfm = load("ref_triton_fused_moe", "grouped_gemm_opt/triton_fused_moe.py")
    for name, counts in EDGE_CASES.items():
        x, w, tpe = edge_inputs(counts)
        xf, wf = x.float(), w.float()
        y = tgg.triton_grouped_gemm(xf, wf, tpe, BLOCK_M=32, BLOCK_N=32, BLOCK_K=32)
        yf = tfm.triton_fused_moe(xf, wf, tpe, BLOCK_M=32, BLOCK_N=32, BLOCK_K=32)
        for tag, t in (("tgg", y), ("tfm", yf)):
            out[f"{tag}_{name}_row_sum"] = t.double().sum(1).numpy()
            out[f"{tag}_{name}_col_sum"] = t.double().sum(0).numpy()
            out[f"{tag}_{name}_sample"] = t.reshape(-1)[::37].numpy()

    # routing generators
    for T, E in [(4096, 8), (8192, 64), (1000, 7), (16384, 256)]:
        out[f"uniform_{T}_{E}"] = ref.uniform_distribution(T, E).numpy()
        out[f"skewed_{T}_{E}"] = ref.skewed_distribution(T, E).numpy()

    np.savez_compressed(HERE / "reference_golden.npz", **out)
    print("wrote", HERE / "reference_golden.npz", sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
