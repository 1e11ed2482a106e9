"""Parity through the C ABI alone (ctypes on libblockfp8_b200.so, no torch ops),
against the CPU oracle, on the Qwen3-8B linear shapes of the benchmark.

Sizes: the four Qwen3-8B linear shapes at decode M (full outputs checked
against the oracle) and at prefill M (a row sample against the oracle, plus
the size-independent property that each output row depends only on its own
input row: the first rows of a large call equal a small call bitwise).
"""

import numpy as np
import pytest
import torch

from blockfp8_b200 import _native, capi
from helpers import (FP8, assert_close, assert_exact, bf16_activations, codes, f32,
                     integer_operands, oracle_gemm, oracle_quant, token_limit)
from oracle import oracle as O

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

DEV = "cuda"
SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (24576, 4096), "down": (4096, 12288)}


def _weights(n, k, seed=0):
    """w ~ N(0, 0.02) on a CPU generator, quantized by the oracle."""
    g = torch.Generator().manual_seed(seed)
    b, sb = O.quantize_weights((torch.randn(n, k, generator=g) * 0.02).numpy())
    return b, sb, torch.from_numpy(b).view(FP8).to(DEV), torch.from_numpy(sb).to(DEV)


def test_library_reports_itself():
    lib = _native.capi()
    assert lib.bfp8_abi_version() == 1
    assert lib.bfp8_num_configs() >= 1
    assert capi.choose_plan(1, 6144, 4096, 148).splits != 0  # decode: stream-K over the SMs


@pytest.mark.parametrize("m", [1, 7, 33])
def test_quantize_through_c_abi(m):
    x = bf16_activations(m, 4096, seed=m, ties=m == 7)
    q, s = capi.quantize(x.to(DEV))
    q2, s2 = oracle_quant(x)
    assert np.array_equal(codes(q), q2) and np.array_equal(f32(s), s2)


@pytest.mark.parametrize("layer", sorted(SHAPES))
@pytest.mark.parametrize("m", [1, 2, 4, 8, 16, 32])
def test_decode_shapes_full_output(layer, m):
    n, k = SHAPES[layer]
    b_np, sb_np, b, sb = _weights(n, k, seed=1)
    x = bf16_activations(m, k, seed=100 + m, scale=1.0)
    q, s = capi.quantize(x.to(DEV))
    c = capi.gemm(q, s, b, sb)
    a_np, sa_np = oracle_quant(x)
    assert np.array_equal(codes(q), a_np)
    assert_close(c, O.reference_gemm(a_np, sa_np, b_np, sb_np))
    # the fused route gives the same bits under the same plan
    assert torch.equal(capi.gemm(x.to(DEV), None, b, sb, fused=True), c)


@pytest.mark.parametrize("layer", sorted(SHAPES))
def test_prefill_shapes_row_sample_and_row_independence(layer):
    n, k = SHAPES[layer]
    m = 4096 if layer != "gate_up" else 8192
    b_np, sb_np, b, sb = _weights(n, k, seed=2)
    x = bf16_activations(m, k, seed=7, scale=1.0).to(DEV)
    q, s = capi.quantize(x)
    c = capi.gemm(q, s, b, sb)
    rows = np.r_[0:64, m - 64:m, np.random.default_rng(0).integers(0, m, 64)]
    a_np = codes(q)[rows]
    sa_np = f32(s)[rows]
    assert_close(c[torch.from_numpy(rows).to(DEV)], O.reference_gemm(a_np, sa_np, b_np, sb_np))
    # Each output row depends only on its own activation row: under the
    # large call's plan, a 256-row call reproduces its first rows bitwise.
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    plan = capi.choose_plan(m, n, k, sms)
    c_small = capi.gemm(q[:256], s[:256], b, sb, config=plan.config, splits=plan.splits)
    assert torch.equal(c[:256], c_small)


@pytest.mark.parametrize("splits", [1, 2, 5])
def test_exact_integer_through_c_abi(splits):
    a, sa, b, sb = integer_operands(77, 1032, 1040, seed=splits)
    assert_exact(capi.gemm(a, sa, b, sb, config=1, splits=splits), oracle_gemm(a, sa, b, sb))


def test_bad_arguments_come_back_as_errors():
    a, sa, b, sb = integer_operands(4, 256, 256)
    c = torch.empty(4, 256, dtype=torch.bfloat16, device=DEV)
    p = capi.problem(a, sa, b, sb, c)
    p.K = 200  # not a multiple of 16
    with pytest.raises(RuntimeError, match="K must be"):
        capi.launch_gemm(p, capi.choose_plan(4, 256, 256, 148))
    p = capi.problem(a, sa, b, sb, c)
    plan = capi.choose_plan(4, 256, 256, 148)
    plan.config = 99
    with pytest.raises(RuntimeError, match="config"):
        capi.launch_gemm(p, plan)


# ---- the two fused modes --------------------------------------------------------

IN_GEMM_CASES = [
    (1, 24576, 2048 + 128, 3),   # 192 tiles x 3 ragged splits: several units per CTA, short last split
    (5, 4096, 4096, 1),          # one split of 32 K blocks: fits only the 16-token tiles
    (17, 6144, 4096 + 16, 4),    # ragged K tail, tokens past one tile
    (33, 2048, 12288, 12),       # down-like K
    (64, 1024, 4096, 8),
    (1, 24576, 4096, -148),      # stream-K: 41-42 K blocks per CTA across tile boundaries
    (16, 4096, 12288, -148),
    (7, 6144, 4096, -37),
]


@pytest.mark.parametrize("m, n, k, splits", IN_GEMM_CASES)
def test_both_fused_modes_equal_the_quantized_gemm(m, n, k, splits):
    """Quantization inside the GEMM (fused mode 2) and the quantization kernel
    + GEMM (mode 1) give the pre-quantized GEMM's bits under every
    configuration; mode 2 falls back to mode 1 where the plan's K range does
    not fit the resident operand or the configuration has no such variant."""
    b_np, sb_np, b, sb = _weights(n, k, seed=3)
    x = bf16_activations(m, k, seed=7 + m, ties=True).to(DEV)
    q, s = capi.quantize(x)
    lib = _native.capi()
    names = [lib.bfp8_config_name(i).decode() for i in range(lib.bfp8_num_configs())]
    for config in range(lib.bfp8_num_configs()):
        if splits < 0 and names[config].startswith("m256"):
            continue  # CTA pairs have no stream-K schedule
        if (token_limit(names[config]) or m) < m:
            continue  # more tokens than a weight-streaming tile holds
        expect = capi.gemm(q, s, b, sb, config=config, splits=splits)
        for mode in (1, 2):
            got = capi.gemm(x, None, b, sb, config=config, splits=splits, fused=mode)
            assert torch.equal(got, expect), (config, mode)
    a_np, sa_np = oracle_quant(x.cpu())
    assert_close(expect, O.reference_gemm(a_np, sa_np, b_np, sb_np))
    assert _native.device_status(reset=True) == 0


def test_roofline_probes_answer_in_range():
    """The in-library probes: dense e4m3 MMA rate near the 8192 multiply-adds
    per clock per SM of the tensor core, and an HBM read rate of several TB/s."""
    tf, mpc = _native.probe_mma(256, 500)
    assert 6000 < mpc <= 8200 and tf > 1500, (tf, mpc)
    buf = torch.empty(2 << 30, dtype=torch.uint8, device=DEV)
    gbs = _native.probe_hbm_read(buf, reps=3)
    del buf
    assert 3000 < gbs < 9000, gbs
    assert _native.device_status(reset=True) == 0
