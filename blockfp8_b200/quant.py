"""Block quantization to float8_e4m3fn in plain PyTorch (any device).

Part of the public API the reference exports (blockfp8/quant.py:39-79):
quantize_weights prepares B operands (checkpoints ship them already
quantized); quantize_activations is the readable statement of what the CUDA
quantizer (quantize_cuda / the linear op) computes.  Neither is on the CUDA
hot path, and nothing on that path falls back to them.

    scale = max(amax(|block|), eps) / 448      true float32 division
    q     = e4m3(clamp(x / scale, -448, 448))  round to nearest even

torch divides by a Python scalar as a multiply by its reciprocal, which is one
ulp off amax / 448 for a few percent of groups, so the division below is
tensor by tensor.
"""

import torch
import torch.nn.functional as F

from .layout import BLOCK_N, FP8_DTYPE, FP8_MAX, GROUP_K, cdiv


def _block_amax(xf: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """amax(|x|) over [rows x cols] blocks; ragged edge blocks are zero-padded."""
    m, k = xf.shape
    mb, kb = cdiv(m, rows), cdiv(k, cols)
    padded = F.pad(xf.abs(), (0, kb * cols - k, 0, mb * rows - m))
    return padded.view(mb, rows, kb, cols).amax(dim=3).amax(dim=1)


def _scales(amax: torch.Tensor, eps: float) -> torch.Tensor:
    floored = amax.clamp_min(eps)
    return torch.div(floored, torch.full_like(floored, FP8_MAX))


def _to_fp8(xf: torch.Tensor, s_full: torch.Tensor) -> torch.Tensor:
    return torch.div(xf, s_full).clamp(-FP8_MAX, FP8_MAX).to(FP8_DTYPE)


def quantize_activations(
    x: torch.Tensor,
    group_size: int = GROUP_K,
    eps: float = 1e-10,
    column_major_scales: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
    """x [M, K] -> (x_q [M, K] float8_e4m3fn, scales [M, ceil(K/128)] float32).

    One scale per row per 128-wide K group; the last group may be narrower.
    column_major_scales=True (default) returns M-contiguous scales, strides
    (1, M), the layout quantize_cuda writes.
    """
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D [M, K], got shape {tuple(x.shape)}")
    if group_size != GROUP_K:
        raise ValueError(f"only group_size={GROUP_K} is supported, got {group_size}")
    k = x.shape[1]
    xf = x.float()
    scales = _scales(_block_amax(xf, 1, GROUP_K), eps)
    x_q = _to_fp8(xf, scales.repeat_interleave(GROUP_K, dim=1)[:, :k])
    if column_major_scales:
        scales = scales.t().contiguous().t()
    return x_q, scales


def quantize_weights(w: torch.Tensor, eps: float = 1e-10) -> tuple[torch.Tensor, torch.Tensor]:
    """w [N, K] -> (w_q [N, K] float8_e4m3fn, scales [ceil(N/128), ceil(K/128)] float32)."""
    if w.dim() != 2:
        raise ValueError(f"w must be 2-D [N, K], got shape {tuple(w.shape)}")
    n, k = w.shape
    wf = w.float()
    scales = _scales(_block_amax(wf, BLOCK_N, GROUP_K), eps)
    s_full = scales.repeat_interleave(BLOCK_N, dim=0)[:n].repeat_interleave(GROUP_K, dim=1)[:, :k]
    return _to_fp8(wf, s_full), scales.contiguous()
