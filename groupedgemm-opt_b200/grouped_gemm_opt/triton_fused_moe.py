"""``triton_fused_moe`` kept as a name for drop-in compatibility with the reference
(grouped_gemm_opt/triton_fused_moe.py:104-150). Its semantics there are the plain grouped GEMM
over expert-sorted rows (identity gather/scatter), so it runs the tcgen05 grouped GEMM. Unlike the
reference kernel it stays correct when a 128-row tile spans more than four experts.
For the full MoE layer (router, permute, SwiGLU, down projection, combine) use ``fused_moe``.
"""
import torch

from grouped_gemm_opt.ops import TileConfig, grouped_gemm_opt


def triton_fused_moe(
    input: torch.Tensor,
    weights: torch.Tensor,
    tokens_per_expert: torch.Tensor,
    BLOCK_M: int = 128,
    BLOCK_N: int = 128,
    BLOCK_K: int = 64,
) -> torch.Tensor:
    """Fused-MoE GEMM with the reference's arguments: ``out[i] = input[i] @ W[e(i)].T``."""
    if input.size(0) == 0:
        return torch.empty(0, weights.size(1), device=input.device, dtype=input.dtype)
    tc = TileConfig.Co_128x256x64 if BLOCK_N >= 256 else TileConfig.Co_128x128x64
    return grouped_gemm_opt(input, weights, tokens_per_expert, tc, sort_by_m=False)
