"""The activation quantizer's fast arithmetic against the reference's, on the
whole input domain (GPU).

The kernels quantize x / scale as x * r with one correction step (r the
correctly rounded reciprocal of the scale) instead of one IEEE division per
value.  The reference's sequence (blockfp8/quant.py:25-64,
csrc/quant_sm89.cu:38-59) divides.  Their codes must be identical.  x is
bf16 and the group amax is eps or a bf16 magnitude, so the domain is small:
bfp8_probe_quantizer runs both paths on every (amax, x) pair with |x| <=
amax -- about 10^9 of them -- on the GPU and counts the codes that differ.
The scale amax / 448 is formed the same way (a product with RN(1/448) and
one correction step); bfp8_probe_scale compares it with the division on
every finite non-negative float.
"""

import pytest
import torch

import blockfp8
from blockfp8_b200 import _native

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]


def test_fast_scale_equals_division_on_every_float():
    assert blockfp8.native_available(), "native libraries not built"
    bad, first = _native.probe_scale()
    assert bad == 0, f"{bad} scales differ; first at amax bits {first - 1:#x}"
    assert _native.device_status(reset=True) == 0


@pytest.mark.parametrize("eps", [1e-10, 1e-4, 0.5])
def test_fast_quantization_equals_division_on_every_input(eps):
    assert blockfp8.native_available(), "native libraries not built"
    bad, first = _native.probe_quantizer(eps)
    assert bad == 0, f"{bad} codes differ; first at amax bits {first >> 32:#x}, x bits {(first & 0xFFFFFFFF) - 1:#x}"
    assert _native.device_status(reset=True) == 0
