"""The no-allocation GEMM entry point, through the C ABI.

bfp8_launch_gemm_noalloc serves callers that cannot allocate device memory
on their path (a serving loop whose memory is reserved up front, an FFI host
without a CUDA allocator): it takes its split-K and fused-path scratch from
a fixed array inside the library instead of a caller-provided workspace.
These tests check that it gives the same output as bfp8_launch_gemm with an
allocated workspace, on two calls in a row (the second reuses the array the
first left behind), and that a plan too large for the array is refused.

This file is collected last on purpose, so a failure here comes after every
other test has run; it also passes on its own in a fresh process.
"""

import ctypes

import pytest
import torch

from blockfp8_b200 import _native, capi
from helpers import assert_close, bf16_activations, oracle_gemm, realistic_operands

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

DEV = "cuda"


def _noalloc(p, plan):
    lib = _native.capi()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _native.check(lib.bfp8_launch_gemm_noalloc(ctypes.byref(p), plan, stream))


def _names():
    lib = _native.capi()
    return [lib.bfp8_config_name(i).decode() for i in range(lib.bfp8_num_configs())]


@pytest.mark.parametrize("m, n, k, config, splits, fused", [
    (16, 6144, 4096, "w128t16s10", 3, False),   # decode, swapped tiles, split-K
    (37, 392, 2064, "m128n128s6", 7, False),    # tails in every dimension
    (300, 1024, 4096, "m128n256s4", 4, False),  # prefill tiles, split-K
    (4, 4096, 4096, "w128t16s10", 8, True),     # fused quantization + split-K
])
def test_noalloc_matches_the_workspace_entry_point_twice(m, n, k, config, splits, fused):
    names = _names()
    plan = _native.Plan(names.index(config), splits, 1 if fused else 0)
    if fused:
        x = bf16_activations(m, k, seed=5).to(DEV)
        _, _, b, sb = realistic_operands(1, n, k, seed=6)
        a, sa = x, None
    else:
        a, sa, b, sb = realistic_operands(m, n, k, seed=splits)
    ref_c = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    p_ref = capi.problem(a, sa, b, sb, ref_c)
    assert _native.capi().bfp8_counters_needed(ctypes.byref(p_ref), plan) > 0  # scratch is used
    ws, cnt = capi.scratch(p_ref, plan, a.device)
    capi.launch_gemm(p_ref, plan, ws, cnt)

    for call in range(2):
        c = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=DEV)
        _noalloc(capi.problem(a, sa, b, sb, c), plan)
        torch.cuda.synchronize()
        assert torch.equal(c, ref_c), f"call {call} differs from bfp8_launch_gemm"
    if not fused:
        assert_close(c, oracle_gemm(a, sa, b, sb))
    assert _native.device_status(reset=True) == 0


def test_noalloc_refuses_plans_larger_than_its_scratch():
    names = _names()
    a = torch.zeros(8192, 4096, device=DEV).to(torch.float8_e4m3fn)
    b = torch.zeros(24576, 4096, device=DEV).to(torch.float8_e4m3fn)
    sa = torch.ones(32, 8192, device=DEV).t()
    sb = torch.ones(192, 32, device=DEV)
    c = torch.empty(8192, 24576, dtype=torch.bfloat16, device=DEV)
    plan = _native.Plan(names.index("m128n256s4"), 8, 0)  # ~1.6 GB of split-K partials
    with pytest.raises(RuntimeError, match="fixed scratch holds"):
        _noalloc(capi.problem(a, sa, b, sb, c), plan)
