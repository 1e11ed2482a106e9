"""Python entry points of the B200 block-FP8 linear path.

Same names, arguments, return values and errors as the reference's API
(simon-jd/blockfp8 blockfp8/gemm.py:13-203): ValueError for arguments the
kernels cannot take (with the same reasons), RuntimeError when the native
library is missing, CPU tensors pointed at reference_gemm.  Every compute
entry point goes through torch.ops.blockfp8.* (csrc/ops.cpp) into the sm_100a
kernels; there is no other implementation to fall back to.
"""

import torch

from . import _native
from .layout import BLOCK_N, FP8_DTYPE, GROUP_K, K_ALIGN, N_ALIGN, cdiv

_LIB = _native.OPS_LIB


def native_available() -> bool:
    """True once the native libraries (_C.so over libblockfp8_b200.so) are loaded."""
    return _native.load_ops()


def _require_native() -> None:
    if not native_available():
        raise RuntimeError(f"native extension not built ({_LIB} missing); "
                           "run python -m blockfp8_b200.build")


def check_gemm_args(
    a_q: torch.Tensor,
    a_scales: torch.Tensor,
    b_q: torch.Tensor,
    b_scales: torch.Tensor,
    out_dtype: torch.dtype,
) -> tuple[int, int, int]:
    """Validate shapes, dtypes and alignment; returns (M, N, K).

    Raises ValueError with the reason for anything the kernels cannot take.
    """
    for name, t in (("a_q", a_q), ("b_q", b_q)):
        if t.dtype != FP8_DTYPE:
            raise ValueError(f"{name} must be float8_e4m3fn, got {t.dtype}")
        if t.dim() != 2:
            raise ValueError(f"{name} must be 2-D, got shape {tuple(t.shape)}")
    m, k = a_q.shape
    n, k_b = b_q.shape
    if k != k_b:
        raise ValueError(f"K mismatch: a_q is [{m}, {k}], b_q is [{n}, {k_b}]")
    if k == 0 or k % K_ALIGN:
        raise ValueError(f"K must be a positive multiple of {K_ALIGN}, got {k}")
    if n == 0 or n % N_ALIGN:
        raise ValueError(f"N must be a positive multiple of {N_ALIGN}, got {n}")
    for name, t in (("a_q", a_q), ("b_q", b_q)):
        if t.stride(1) != 1 or t.stride(0) % K_ALIGN:
            raise ValueError(f"{name} must be row-major with a row stride that is a multiple of "
                             f"{K_ALIGN} elements, got strides {t.stride()}")
        if t.data_ptr() % 16:
            raise ValueError(f"{name} must be 16-byte aligned")
    kb, nb = cdiv(k, GROUP_K), cdiv(n, BLOCK_N)
    if a_scales.dtype != torch.float32 or tuple(a_scales.shape) != (m, kb):
        raise ValueError(f"a_scales must be float32 [{m}, {kb}], "
                         f"got {a_scales.dtype} {tuple(a_scales.shape)}")
    if b_scales.dtype != torch.float32 or tuple(b_scales.shape) != (nb, kb):
        raise ValueError(f"b_scales must be float32 [{nb}, {kb}], "
                         f"got {b_scales.dtype} {tuple(b_scales.shape)}")
    devices = {t.device for t in (a_q, a_scales, b_q, b_scales)}
    if len(devices) != 1:
        raise ValueError(f"all operands must be on one device, got {sorted(map(str, devices))}")
    if out_dtype != torch.bfloat16:
        raise ValueError(f"out_dtype must be torch.bfloat16, got {out_dtype}")
    return m, n, k


def gemm(
    a_q: torch.Tensor,
    a_scales: torch.Tensor,
    b_q: torch.Tensor,
    b_scales: torch.Tensor,
    out_dtype: torch.dtype = torch.bfloat16,
    *,
    config: int = -1,
    split_k: int = 0,
) -> torch.Tensor:
    """C [M, N] bf16 = block-scaled A_q [M, K] @ B_q [N, K]^T (layouts in
    blockfp8_b200.layout).  config / split_k override the planner's choice
    (-1 / 0 = automatic; split_k < 0 = stream-K over -split_k CTAs);
    configs() lists the compiled configurations."""
    m, n, _ = check_gemm_args(a_q, a_scales, b_q, b_scales, out_dtype)
    if not a_q.is_cuda:
        raise ValueError("gemm runs on CUDA tensors only; use blockfp8.reference_gemm on CPU")
    _require_native()
    if m == 0:
        return torch.empty(0, n, dtype=out_dtype, device=a_q.device)
    return torch.ops.blockfp8.gemm(a_q, a_scales, b_q, b_scales, config, split_k)


def gemm_bf16(
    x: torch.Tensor,
    b_q: torch.Tensor,
    b_scales: torch.Tensor,
    *,
    eps: float = 1e-10,
    config: int = -1,
    split_k: int = 0,
) -> torch.Tensor:
    """C [M, N] bf16 = x [M, K] bf16 @ B^T with x quantized as part of the
    call, exactly as quantize_activations(x, eps=eps) does, so the result is
    bitwise gemm(*quantize_activations(x), b_q, b_scales) under the same plan.
    config / split_k index fused_configs()."""
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise ValueError(f"x must be 2-D bfloat16, got {x.dtype} {tuple(x.shape)}")
    if x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        raise ValueError(f"x must be row-major, 16-byte aligned rows; got strides {x.stride()}")
    m, k = x.shape
    if b_q.dtype != FP8_DTYPE or b_q.dim() != 2 or b_q.shape[1] != k:
        raise ValueError(f"b_q must be float8_e4m3fn [N, {k}], got {b_q.dtype} {tuple(b_q.shape)}")
    if k % K_ALIGN or b_q.shape[0] % N_ALIGN:
        raise ValueError(f"K must be a multiple of {K_ALIGN} and N of {N_ALIGN}")
    nb, kb = cdiv(b_q.shape[0], BLOCK_N), cdiv(k, GROUP_K)
    if b_scales.dtype != torch.float32 or tuple(b_scales.shape) != (nb, kb):
        raise ValueError(f"b_scales must be float32 [{nb}, {kb}]")
    if not x.is_cuda:
        raise ValueError("gemm_bf16 runs on CUDA tensors only")
    _require_native()
    return torch.ops.blockfp8.gemm_bf16(x, b_q, b_scales, config, split_k, eps)


def prefers_fused(m: int, n: int, k: int) -> bool:
    """Whether linear runs this shape through gemm_bf16 (the fused plan table)."""
    _require_native()
    return torch.ops.blockfp8.prefers_fused(m, n, k)


def _check_bf16(x: torch.Tensor) -> None:
    if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_cuda:
        raise ValueError(f"x must be a 2-D bfloat16 CUDA tensor, got {x.dtype} {tuple(x.shape)}")
    if x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        raise ValueError(f"x must be row-major, 16-byte aligned rows; got strides {x.stride()}")
    if x.shape[1] == 0 or x.shape[1] % K_ALIGN:
        raise ValueError(f"K must be a positive multiple of {K_ALIGN}, got {x.shape[1]}")
    _require_native()


def quantize_cuda(x: torch.Tensor, eps: float = 1e-10) -> tuple[torch.Tensor, torch.Tensor]:
    """The CUDA activation quantizer: bitwise quantize_activations(x, eps)
    for bf16 x; scales are M-contiguous, strides (1, M)."""
    _check_bf16(x)
    return torch.ops.blockfp8.quantize(x, eps)


def linear(x: torch.Tensor, b_q: torch.Tensor, b_scales: torch.Tensor) -> torch.Tensor:
    """bf16 x [M, K] @ block-FP8 weight^T in one call: quantize_cuda then gemm
    (gemm_bf16 where prefers_fused).  This is what the vLLM plugin runs."""
    _check_bf16(x)
    return torch.ops.blockfp8.linear(x, b_q, b_scales)


def configs() -> list[str]:
    """Names of the compiled kernel configurations, indexed by config id."""
    _require_native()
    return torch.ops.blockfp8.config_names().split(";")


def fused_configs() -> list[str]:
    """Names of the fused-quantization configurations (gemm_bf16)."""
    _require_native()
    return torch.ops.blockfp8.fused_config_names().split(";")
