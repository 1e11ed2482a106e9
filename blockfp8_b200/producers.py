"""The layers that feed a block-FP8 linear, emitting its e4m3 operand.

`rms_norm_quant` (RMSNorm, optionally after the residual add) and
`silu_mul_quant` (SiLU-and-mul) return the codes and M-major scales that
`blockfp8.gemm` takes, from one kernel each: the linear after them then runs
the GEMM alone, with no quantization launch and no bf16 activation written
to and read back from HBM.  Their codes and scales equal `quantize_cuda`
applied to the bf16 output the unfused layer would produce (tests check it
bit for bit); `rms_norm` / `silu_mul` return that bf16 output from the same
kernels.

No reference counterpart: the reference quantizes activations in a kernel
of its own before every GEMM (csrc/quant_sm89.cu) and leaves fusion into the
previous layer outside its kernels (docs/design-tradeoffs.md:158-160).
"""

import ctypes

import torch

from . import _native
from ._native import RmsNormQuantProblem, SiluMulQuantProblem, check

__all__ = ["rms_norm_quant", "silu_mul_quant", "rms_norm", "silu_mul"]


def _ops():
    if not _native.load_ops():
        raise RuntimeError("blockfp8_b200 native library not built: run python -m blockfp8_b200.build")
    return torch.ops.blockfp8_b200


def rms_norm_quant(x: torch.Tensor, weight: torch.Tensor, variance_epsilon: float,
                   residual: torch.Tensor | None = None, eps: float = 1e-10):
    """(q [M, H] e4m3, scales [M, H/128] M-major, h) of RMSNorm(x [+ residual]).

    h is x + residual in bf16 (the next layer's residual) when a residual is
    given, else an empty tensor."""
    return _ops().rms_norm_quant(x, weight, variance_epsilon, residual, eps)


def silu_mul_quant(x: torch.Tensor, eps: float = 1e-10):
    """(q [M, I] e4m3, scales [M, I/128] M-major) of silu(x[:, :I]) * x[:, I:]."""
    return _ops().silu_mul_quant(x, eps)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, variance_epsilon: float,
             residual: torch.Tensor | None = None):
    """The bf16 RMSNorm output of the same kernel (and x + residual when a
    residual is given), through the C ABI; for comparisons and for timing the
    unfused layer."""
    m, h = x.shape
    y = torch.empty_like(x)
    h_out = torch.empty_like(x) if residual is not None else None
    p = RmsNormQuantProblem()
    p.x, p.ldx = x.data_ptr(), x.stride(0)
    if residual is not None:
        p.residual, p.ldr = residual.data_ptr(), residual.stride(0)
        p.residual_out, p.ldro = h_out.data_ptr(), h_out.stride(0)
    p.weight = weight.data_ptr()
    p.y, p.ldy = y.data_ptr(), y.stride(0)
    p.M, p.H, p.variance_epsilon, p.eps = m, h, variance_epsilon, 1e-10
    check(_native.capi().bfp8_launch_rmsnorm_quant(ctypes.byref(p),
                                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return (y, h_out) if residual is not None else y


def silu_mul(x: torch.Tensor) -> torch.Tensor:
    """The bf16 SiLU-and-mul output of the same kernel, through the C ABI."""
    m, i = x.shape[0], x.shape[1] // 2
    y = torch.empty(m, i, dtype=torch.bfloat16, device=x.device)
    p = SiluMulQuantProblem()
    p.x, p.ldx = x.data_ptr(), x.stride(0)
    p.y, p.ldy = y.data_ptr(), y.stride(0)
    p.M, p.I, p.eps = m, i, 1e-10
    check(_native.capi().bfp8_launch_silu_mul_quant(ctypes.byref(p),
                                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return y
