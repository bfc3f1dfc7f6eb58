"""grouped_gemm_opt -- B200-native (sm_100a) MoE grouped GEMM and fused MoE layer.

Drop-in for the reference package's API (grouped_gemm_opt/__init__.py:1-5) plus ``fused_moe``.
"""
from grouped_gemm_opt.ops import (TileConfig, check_device_errors, grouped_gemm_opt,
                                  grouped_gemm_opt_fp8, grouped_gemm_opt_host,
                                  grouped_gemm_opt_mxfp8, mxfp8_block_gate_up, quantize_fp8,
                                  quantize_mxfp8)
from grouped_gemm_opt.triton_fused_moe import triton_fused_moe
from grouped_gemm_opt.triton_grouped_gemm import triton_grouped_gemm
from grouped_gemm_opt.moe import (EPBuffers, MoEFP8Weights, MoEMXFP8Weights, StageEvents,
                                  MoEHostPipeline, fused_moe, fused_moe_fp8, fused_moe_host,
                                  fused_moe_mxfp8,
                                  quantize_moe_weights, quantize_moe_weights_mxfp8)

__all__ = ["grouped_gemm_opt", "TileConfig", "triton_fused_moe", "triton_grouped_gemm",
           "fused_moe", "check_device_errors", "grouped_gemm_opt_host", "EPBuffers",
           "grouped_gemm_opt_fp8", "quantize_fp8", "fused_moe_fp8", "quantize_moe_weights",
           "MoEFP8Weights", "quantize_mxfp8", "grouped_gemm_opt_mxfp8", "mxfp8_block_gate_up",
           "fused_moe_mxfp8", "quantize_moe_weights_mxfp8", "MoEMXFP8Weights",
           "fused_moe_host", "MoEHostPipeline", "StageEvents"]
