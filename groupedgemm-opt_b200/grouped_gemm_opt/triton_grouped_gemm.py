"""``triton_grouped_gemm`` kept as a name for drop-in compatibility with the reference
(grouped_gemm_opt/triton_grouped_gemm.py:139-197). There is no Triton here: the call runs the
tcgen05 grouped GEMM; BLOCK_N picks the tile width, the other block arguments are accepted hints.
"""
import torch

from grouped_gemm_opt.ops import TileConfig, grouped_gemm_opt


def triton_grouped_gemm(
    input: torch.Tensor,
    weights: torch.Tensor,
    tokens_per_expert: torch.Tensor,
    BLOCK_M: int = 128,
    BLOCK_N: int = 128,
    BLOCK_K: int = 64,
    num_warps: int = 4,
    num_stages: int = 3,
) -> torch.Tensor:
    """Grouped GEMM, one expert per tile. Same arguments and result as the reference."""
    if input.size(0) == 0:
        return torch.empty(0, weights.size(1), device=input.device, dtype=input.dtype)
    tc = TileConfig.Co_128x256x64 if BLOCK_N >= 256 else TileConfig.Co_128x128x64
    return grouped_gemm_opt(input, weights, tokens_per_expert, tc, sort_by_m=False)
