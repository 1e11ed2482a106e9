"""Block-scaled FP8 linear layers on NVIDIA B200 (sm_100a).

A from-scratch B200 implementation of blockfp8's hot path (per-token 1x128
e4m3 activation quantizer + 128x128 block-scaled FP8 GEMM with tcgen05 MMAs
into tensor memory), behind the reference's Python API, torch op schemas and
vLLM plugin entry point.  `import blockfp8` gives the same module.
"""

from .gemm import (
    check_gemm_args,
    configs,
    fused_configs,
    gemm,
    gemm_bf16,
    linear,
    native_available,
    prefers_fused,
    quantize_cuda,
)
from .layout import BLOCK_N, FP8_DTYPE, FP8_MAX, GROUP_K
from .quant import quantize_activations, quantize_weights
from .reference import dequantize_activations, dequantize_weights, error_bound, reference_gemm

__all__ = [
    "BLOCK_N",
    "FP8_DTYPE",
    "FP8_MAX",
    "GROUP_K",
    "check_gemm_args",
    "configs",
    "dequantize_activations",
    "dequantize_weights",
    "error_bound",
    "fused_configs",
    "gemm",
    "gemm_bf16",
    "linear",
    "native_available",
    "prefers_fused",
    "quantize_activations",
    "quantize_cuda",
    "quantize_weights",
    "reference_gemm",
]
