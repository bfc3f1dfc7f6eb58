"""Python API of the grouped GEMM, a drop-in for the reference's grouped_gemm_opt/ops.py.

Same names, argument meaning, defaults and error behaviour as the reference
(grouped_gemm_opt/ops.py:8-84); the work runs in the persistent tcgen05 kernel of
libggo_b200.so through the ``_C`` binding.
"""
from enum import IntEnum

import torch

from grouped_gemm_opt._native import _C


class TileConfig(IntEnum):
    """Tile configuration, value-compatible with the reference enum (ops.py:8-29).

    On B200 the kernel is always a persistent tcgen05 grouped GEMM; the value picks its tile:
      Co_128x128x64 / PP_128x128x128 -- single-CTA 128x128 tile, 6-stage TMA ring
      Co_128x256x64  -- single-CTA 128x256 tile, 4-stage ring
      PP_128x256x64  -- CTA pair (cta_group::2), 256x256 tile (+ a pass over short tails)
      AUTO        -- 128x128 when wider tiles leave SMs idle, the CTA pair when segments
                     average >= 192 rows, else 128x256 (decided without reading the counts)
      CuBLAS_Seq  -- accepted for compatibility; runs the AUTO choice (no library GEMM)
    """
    Co_128x128x64 = 0
    Co_128x256x64 = 1
    PP_128x128x128 = 2
    PP_128x256x64 = 3
    AUTO = 4
    CuBLAS_Seq = 5


class _GroupedGemmFn(torch.autograd.Function):
    """Autograd wrapper: forward = the tcgen05 grouped GEMM; backward = the dgrad kernel
    (dx = dy @ W[e]) and the wgrad kernel (dW[e] = dy_e^T @ x_e). The reference is forward-only;
    this makes the same call usable for training."""

    @staticmethod
    def forward(ctx, input, weights, tokens_per_expert, tile_config, sort_by_m):
        ctx.save_for_backward(input, weights, tokens_per_expert)
        ctx.tile_config, ctx.sort_by_m = tile_config, sort_by_m
        return _C.grouped_gemm_opt_forward(input, weights, tokens_per_expert, tile_config,
                                           sort_by_m)

    @staticmethod
    def backward(ctx, grad_out):
        input, weights, tpe = ctx.saved_tensors
        grad_out = grad_out.contiguous()
        gi = gw = None
        if ctx.needs_input_grad[0]:
            gi = _C.grouped_gemm_dgrad(grad_out, weights, tpe, ctx.tile_config, ctx.sort_by_m)
        if ctx.needs_input_grad[1]:
            gw = _C.grouped_gemm_wgrad(input, grad_out, tpe, ctx.sort_by_m)
        return gi, gw, None, None, None


def grouped_gemm_opt(
    input: torch.Tensor,
    weights: torch.Tensor,
    tokens_per_expert: torch.Tensor,
    tile_config: TileConfig = TileConfig.AUTO,
    sort_by_m: bool = True,
) -> torch.Tensor:
    """MoE grouped GEMM: ``output[i] = input[i] @ weights[expert_of(i)].T``.

    Args:
        input: [total_tokens, K] bf16/fp16, rows sorted by expert.
        weights: [num_experts, N, K] (torch.nn.Linear layout per expert).
        tokens_per_expert: [num_experts] integer tensor on the CPU or the GPU. GPU counts are
            read only by the kernel: the call never synchronises the host.
        tile_config: a TileConfig (AUTO recommended).
        sort_by_m: process experts heaviest-first (a tile-order hint; results are identical).

    Returns:
        output: [total_tokens, N], same dtype as ``input``.

    Differentiable: when ``input`` or ``weights`` requires grad, the backward runs the dgrad and
    wgrad grouped-GEMM kernels.

    Raises AssertionError for non-CUDA operands, wrong ranks and (CPU counts only)
    ``sum(tokens_per_expert) != total_tokens`` -- as the reference (ops.py:57-64) -- and
    RuntimeError for dtype/shape/alignment errors (as the reference's TORCH_CHECKs).
    """
    assert input.is_cuda and weights.is_cuda
    assert input.dim() == 2 and weights.dim() == 3

    tokens_per_expert = tokens_per_expert.to(torch.int64).contiguous()
    if not tokens_per_expert.is_cuda:
        total = int(tokens_per_expert.sum().item())
        assert total == input.size(0), (
            f"sum(tokens_per_expert)={total} != total_tokens={input.size(0)}")
        # Zero-token experts need no host-side filtering (and no weight copy): the kernel skips
        # them while it builds its tile pool.
    if torch.is_grad_enabled() and (input.requires_grad or weights.requires_grad):
        return _GroupedGemmFn.apply(input.contiguous(), weights.contiguous(),
                                    tokens_per_expert.to(input.device), int(tile_config),
                                    sort_by_m)
    return _C.grouped_gemm_opt_forward(
        input.contiguous(),
        weights.contiguous(),
        tokens_per_expert,
        int(tile_config),
        sort_by_m,
    )


def check_device_errors(device: int = 0) -> None:
    """Synchronises and raises RuntimeError if a kernel on the current stream recorded an error
    (count mismatch with GPU counts, negative count, or an expired bounded wait)."""
    code = int(_C.workspace_error(device))
    if code:
        raise RuntimeError(f"grouped_gemm_opt device error code {code}")


def grouped_gemm_opt_host(
    input: torch.Tensor,
    weights: torch.Tensor,
    tokens_per_expert: torch.Tensor,
    out: torch.Tensor = None,
    tile_config: TileConfig = TileConfig.AUTO,
    sort_by_m: bool = True,
    chunks: int = 4,
) -> torch.Tensor:
    """Grouped GEMM on HOST-resident activations: ``out[i] = input[i] @ weights[e(i)].T`` with
    ``input`` and ``out`` in (pinned) host memory and ``weights`` on the GPU.

    The experts are split into ``chunks`` contiguous groups; each group's rows are copied in,
    multiplied and copied back on three streams, so the host->device copy of group i+1, the
    grouped GEMM of group i and the device->host copy of group i-1 overlap. Returns ``out``
    (allocated pinned if not given) after the stream work is enqueued; it is complete once the
    current stream is synchronised (all work is joined back to it).
    """
    assert weights.is_cuda and weights.dim() == 3 and input.dim() == 2
    assert not input.is_cuda, "input must be in host memory (pin it for overlap)"
    if out is None:
        out = torch.empty(input.size(0), weights.size(1), dtype=input.dtype,
                          pin_memory=True)
    return _C.grouped_gemm_host(input.contiguous(), weights.contiguous(),
                                tokens_per_expert, out, int(tile_config), sort_by_m, chunks)


def quantize_fp8(x: torch.Tensor):
    """Row-wise e4m3 quantisation on the GPU: returns (q float8_e4m3fn, scale fp32) with
    x ~= q * scale[..., None]; scale = rowwise max|x| / 448. Weights [E, N, K] quantise per
    output channel (scale [E, N])."""
    return _C.quantize_fp8_rows(x.contiguous())


def grouped_gemm_opt_fp8(
    input_q: torch.Tensor,
    input_scale: torch.Tensor,
    weights_q: torch.Tensor,
    weight_scale: torch.Tensor,
    tokens_per_expert: torch.Tensor,
    tile_config: TileConfig = TileConfig.AUTO,
    sort_by_m: bool = True,
) -> torch.Tensor:
    """FP8 grouped GEMM: ``out[i] = (q_in[i] @ q_w[e(i)].T) * input_scale[i] * weight_scale[e(i)]``
    with e4m3 operands (tcgen05 kind::f8f6f4, fp32 accumulation) and a bf16 result. Use
    :func:`quantize_fp8` to produce the operands and scales."""
    assert input_q.is_cuda and weights_q.is_cuda
    tokens_per_expert = tokens_per_expert.to(torch.int64).contiguous()
    if not tokens_per_expert.is_cuda:
        total = int(tokens_per_expert.sum().item())
        assert total == input_q.size(0), (
            f"sum(tokens_per_expert)={total} != total_tokens={input_q.size(0)}")
    return _C.grouped_gemm_fp8(input_q.contiguous(), input_scale.contiguous().float(),
                               weights_q.contiguous(), weight_scale.contiguous().float(),
                               tokens_per_expert, int(tile_config), sort_by_m)


def quantize_mxfp8(x: torch.Tensor, tokens_per_expert: torch.Tensor = None):
    """MX e4m3 quantisation on the GPU in the OCP microscaling layout: every 32 consecutive
    elements of a row share one UE8M0 scale 2^(byte - 127). The scale rule is non-saturating
    (X = floor(log2 amax) - 8, plus one when the mantissa of amax exceeds 1.75, so no element
    clips); the OCP MX v1.0 rule (floor(log2 amax) - 8 and clamping) can give a scale one lower.
    Returns (q float8_e4m3fn, scales uint8) with the scales
    in the 128x4 blocked layout the block-scaled tensor cores read, each expert's rows starting a
    fresh 128-row block. Activations [T, K]: pass ``tokens_per_expert`` (the rows are
    expert-sorted). Weights [E, N, K]: leave it None (E segments of N rows). K % 128 == 0."""
    x = x.contiguous()
    if tokens_per_expert is None:
        assert x.dim() == 3, "weights [E, N, K] when tokens_per_expert is None"
        counts = torch.full((x.size(0),), x.size(1), dtype=torch.int64, device=x.device)
    else:
        counts = tokens_per_expert.to(torch.int64)
    return _C.quantize_mxfp8(x, counts)


def grouped_gemm_opt_mxfp8(
    input_q: torch.Tensor,
    input_scale: torch.Tensor,
    weights_q: torch.Tensor,
    weight_scale: torch.Tensor,
    tokens_per_expert: torch.Tensor,
    sort_by_m: bool = True,
) -> torch.Tensor:
    """MXFP8 grouped GEMM: ``out[i] = sum_k (q_in[i,k] 2^s_in[i,k//32]) (q_w[e,n,k] 2^s_w[e,n,k//32])``
    in bf16, the block scales applied by the tensor cores (tcgen05 kind::mxf8f6f4.block_scale,
    fp32 accumulation). Operands and scales come from :func:`quantize_mxfp8` (the input quantised
    with the same ``tokens_per_expert``). Always runs 256 x 256 CTA-pair tiles: there is no tile
    configuration for the MX path."""
    assert input_q.is_cuda and weights_q.is_cuda
    tokens_per_expert = tokens_per_expert.to(torch.int64).contiguous()
    if not tokens_per_expert.is_cuda:
        total = int(tokens_per_expert.sum().item())
        assert total == input_q.size(0), (
            f"sum(tokens_per_expert)={total} != total_tokens={input_q.size(0)}")
    return _C.grouped_gemm_mxfp8(input_q.contiguous(), input_scale.contiguous(),
                                 weights_q.contiguous(), weight_scale.contiguous(),
                                 tokens_per_expert, weights_q.size(0), sort_by_m)


def mxfp8_block_gate_up(w_gate_up: torch.Tensor) -> torch.Tensor:
    """Reorders a gate/up weight [E, 2F, K] (gate rows then up rows) into the blocked layout the
    MXFP8 SwiGLU GEMM reads: [E, 2 * F_pad, K], F_pad = F rounded up to 128, block j = gate rows
    128j..128j+127 then the matching up rows, zero rows past F. A one-time weight preparation."""
    E, two_f, K = w_gate_up.shape
    F = two_f // 2
    rows = _C.mxfp8_glu_rows(F)
    fp = rows // 2
    blk = 128
    out = w_gate_up.new_zeros(E, fp // blk, 2, blk, K)
    g = w_gate_up.new_zeros(E, fp, K)
    g[:, :F] = w_gate_up[:, :F]
    out[:, :, 0] = g.view(E, fp // blk, blk, K)
    g.zero_()
    g[:, :F] = w_gate_up[:, F:]
    out[:, :, 1] = g.view(E, fp // blk, blk, K)
    return out.view(E, rows, K)

