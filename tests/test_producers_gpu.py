"""RMSNorm and SiLU-and-mul that emit the linear's e4m3 operand (GPU).

- The fused codes and scales equal blockfp8.quantize_cuda applied to the
  bf16 output of the same layer (bit for bit), and that bf16 output matches
  a float32 torch statement of the layer (two bf16 steps at most, in a
  small fraction of the values: the row sum is added in another order).
- x + residual comes back exactly as torch's bf16 addition.
- gemm on the fused operand equals linear on the unfused layer's output,
  bit for bit, at decode and prefill M on the Qwen3-8B shapes.
- Infinities and NaN in a group take the quantizer's exact path.
"""

import pytest
import torch

import blockfp8
from blockfp8_b200 import _native, producers

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

DEV = "cuda"


def _rms_ref(h, w, var_eps):
    hf = h.float()
    rstd = torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + var_eps)
    return ((hf * rstd).bfloat16().float() * w.float()).bfloat16()


def _silu_ref(x):
    i = x.shape[1] // 2
    g, u = x[:, :i].float(), x[:, i:].float()
    return ((g / (1 + torch.exp(-g))).bfloat16().float() * u).bfloat16()


def _close_bf16(y, ref, frac=2e-3):
    """Equal, or at most two bf16 steps apart in at most `frac` of the
    values: a row sum added in another order can move bf16(h * rstd) by one
    step, which the product with the weight and its own rounding can turn
    into two."""
    yb, rb = y.view(torch.int16).int(), ref.view(torch.int16).int()
    diff = (yb - rb).abs()
    assert diff.max().item() <= 2, diff.max().item()
    assert (diff != 0).float().mean().item() <= frac


def _same_quant(q, s, y):
    q2, s2 = blockfp8.quantize_cuda(y)
    assert torch.equal(q.view(torch.uint8), q2.view(torch.uint8))
    assert torch.equal(s, s2) and s.stride() == (1, y.shape[0])


@pytest.mark.parametrize("h", [128, 4096, 5120, 16384])
@pytest.mark.parametrize("m", [1, 3, 16, 257])
@pytest.mark.parametrize("with_residual", [False, True])
def test_rms_norm_quant(m, h, with_residual):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + h)
    x = (torch.randn(m, h, device=DEV, generator=g) * 3).bfloat16()
    r = torch.randn(m, h, device=DEV, generator=g).bfloat16() if with_residual else None
    w = (torch.rand(h, device=DEV, generator=g) + 0.5).bfloat16()
    q, s, h_out = producers.rms_norm_quant(x, w, 1e-6, r)
    if with_residual:
        y, h2 = producers.rms_norm(x, w, 1e-6, r)
        hh = (x.float() + r.float()).bfloat16()
        assert torch.equal(h_out, hh) and torch.equal(h2, hh)
    else:
        y = producers.rms_norm(x, w, 1e-6)
        hh = x
        assert h_out.numel() == 0
    _close_bf16(y, _rms_ref(hh, w, 1e-6))
    _same_quant(q, s, y)
    assert _native.device_status(reset=True) == 0


@pytest.mark.parametrize("i", [128, 4224, 12288])
@pytest.mark.parametrize("m", [1, 5, 64])
def test_silu_mul_quant(m, i):
    g = torch.Generator(device=DEV).manual_seed(m + i)
    x = (torch.randn(m, 2 * i, device=DEV, generator=g) * 2).bfloat16()
    q, s = producers.silu_mul_quant(x)
    y = producers.silu_mul(x)
    _close_bf16(y, _silu_ref(x))
    _same_quant(q, s, y)
    assert _native.device_status(reset=True) == 0


@pytest.mark.parametrize("m", [1, 4, 16, 300])
def test_fused_operand_feeds_gemm_like_linear(m):
    g = torch.Generator(device=DEV).manual_seed(m)
    hdim, inter = 4096, 12288
    x = torch.randn(m, hdim, device=DEV, generator=g).bfloat16()
    w = (torch.rand(hdim, device=DEV, generator=g) + 0.5).bfloat16()
    wq = torch.randn(2 * inter, hdim, device=DEV, generator=g) * 0.02
    b, sb = blockfp8.quantize_weights(wq)
    q, s, _ = producers.rms_norm_quant(x, w, 1e-6)
    assert torch.equal(blockfp8.gemm(q, s, b, sb), blockfp8.linear(producers.rms_norm(x, w, 1e-6), b, sb))
    act = (torch.randn(m, 2 * inter, device=DEV, generator=g)).bfloat16()
    wd = torch.randn(hdim, inter, device=DEV, generator=g) * 0.02
    bd, sbd = blockfp8.quantize_weights(wd)
    q2, s2 = producers.silu_mul_quant(act)
    assert torch.equal(blockfp8.gemm(q2, s2, bd, sbd), blockfp8.linear(producers.silu_mul(act), bd, sbd))
    assert _native.device_status(reset=True) == 0


def test_non_finite_groups_take_the_exact_path():
    x = torch.randn(4, 2 * 512, device=DEV).bfloat16()
    x[0, 3] = float("inf")     # gate -> silu(inf) = inf
    x[1, 512 + 7] = float("nan")  # up -> nan product
    x[2, 100] = -float("inf")  # silu(-inf) * u = nan (0 * ...) or -0
    q, s = producers.silu_mul_quant(x)
    _same_quant(q, s, producers.silu_mul(x))
    h = torch.randn(2, 256, device=DEV).bfloat16()
    h[1, 5] = float("inf")
    w = torch.ones(256, device=DEV).bfloat16()
    q, s, _ = producers.rms_norm_quant(h, w, 1e-6)
    _same_quant(q, s, producers.rms_norm(h, w, 1e-6))
    assert _native.device_status(reset=True) == 0


def test_bad_shapes_are_rejected():
    with pytest.raises(RuntimeError, match="multiple of 128"):
        producers.rms_norm_quant(torch.zeros(2, 208, device=DEV).bfloat16(), torch.ones(208, device=DEV).bfloat16(),
                                 1e-6)
    with pytest.raises(RuntimeError, match="I a multiple of 128"):
        producers.silu_mul_quant(torch.zeros(2, 400, device=DEV).bfloat16())
