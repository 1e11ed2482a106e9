"""GPU parity tests of the sm_100a GEMM and quantizer against the CPU oracle.

Restates the semantics of the reference's GPU tests (simon-jd/blockfp8
tests/test_gemm_gpu.py): exact integer cases for every configuration, tail
shape and split count; realistic operands within the parity tolerance
(rel 1e-2 / abs 1e-2 x max|ref|); adversarial scales and values; determinism;
CUDA graphs; fused == quantize-then-GEMM bitwise; the quantizer bit-exact.
The oracle (oracle/) replaces the reference's torch FP64 reference.
"""

import numpy as np
import pytest
import torch

import blockfp8
from helpers import (FP8, assert_close, assert_exact, bf16_activations, codes, f32,
                     integer_operands, oracle_gemm, oracle_quant, realistic_operands, token_limit)
from oracle import oracle as O

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _native():
    # On a GPU box the native libraries must be there: fail, never skip.
    assert blockfp8.native_available(), "native libraries not built"


def _configs():
    return list(range(len(blockfp8.configs()))) if blockfp8.native_available() else [0]


CONFIGS = _configs()


def _pair(config):
    """Configurations on a CTA pair (256-row tiles, cta_group::2)."""
    return blockfp8.native_available() and blockfp8.configs()[config].startswith("m256")


def _tokens(config, m):
    """Skip a weight-streaming configuration for more tokens than it holds
    (it refuses them; decode sizes are covered by the tests below)."""
    lim = token_limit(blockfp8.configs()[config]) if blockfp8.native_available() else None
    if lim is not None and m > lim:
        pytest.skip(f"{blockfp8.configs()[config]} handles at most {lim} tokens")


STREAM = [i for i, n in enumerate(blockfp8.configs()) if token_limit(n)] if blockfp8.native_available() else []

SHAPES = [
    (1, 128, 128),
    (5, 256, 384),
    (16, 512, 1024),
    (33, 264, 272),  # tails in M, N and K
    (64, 384, 2048),
    (130, 136, 4096),
    (257, 1024, 512),
    (300, 520, 144),
]


@pytest.mark.parametrize("config", CONFIGS)
@pytest.mark.parametrize("shape", SHAPES)
def test_exact_integer_case_all_configs(config, shape):
    _tokens(config, shape[0])
    a, sa, b, sb = integer_operands(*shape, seed=sum(shape) % 1000)
    c = blockfp8.gemm(a, sa, b, sb, config=config, split_k=1)
    assert_exact(c, oracle_gemm(a, sa, b, sb))


@pytest.mark.parametrize("config", CONFIGS)
@pytest.mark.parametrize("splits", [2, 3, 7])
def test_exact_integer_case_split_k(config, splits):
    _tokens(config, 37)
    a, sa, b, sb = integer_operands(37, 392, 2048 + 16, seed=splits)
    c = blockfp8.gemm(a, sa, b, sb, config=config, split_k=splits)
    assert_exact(c, oracle_gemm(a, sa, b, sb))


@pytest.mark.parametrize("config", CONFIGS)
@pytest.mark.parametrize("shape, ctas", [((37, 392, 2048 + 16), 148), ((37, 392, 2048 + 16), 5),
                                         ((37, 392, 2048 + 16), 1000), ((1, 24576, 4096), 148),
                                         ((20, 4096, 12288), 148), ((3, 1000, 1040), 7)])
def test_exact_integer_case_stream_k(config, shape, ctas):
    """Stream-K (split_k < 0): CTAs share all tiles' K blocks evenly; tiles cut
    into several parts (ragged, across tile boundaries) sum them in K order."""
    if _pair(config):
        pytest.skip("CTA-pair configurations have no stream-K schedule")
    _tokens(config, shape[0])
    a, sa, b, sb = integer_operands(*shape, seed=ctas % 97)
    c = blockfp8.gemm(a, sa, b, sb, config=config, split_k=-ctas)
    assert_exact(c, oracle_gemm(a, sa, b, sb))


@pytest.mark.parametrize("config", CONFIGS)
def test_stream_k_deterministic_and_in_graph(config):
    if _pair(config):
        with pytest.raises(RuntimeError, match="stream-K"):
            blockfp8.gemm(*realistic_operands(9, 256, 256, seed=8), config=config, split_k=-148)
        return
    a, sa, b, sb = realistic_operands(9, 6144, 4096, seed=8)
    outs = [blockfp8.gemm(a, sa, b, sb, config=config, split_k=-148) for _ in range(3)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    assert_close(outs[0], oracle_gemm(a, sa, b, sb))
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        blockfp8.gemm(a, sa, b, sb, config=config, split_k=-148)
        with torch.cuda.graph(graph, stream=s):
            out = blockfp8.gemm(a, sa, b, sb, config=config, split_k=-148)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):  # the counters are back at zero after every replay
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, outs[0])


@pytest.mark.parametrize("shape", SHAPES + [(1, 4096, 4096), (64, 6144, 4096), (512, 4096, 12288),
                                            (384, 4096, 12288), (768, 6144, 4096)])
def test_realistic_within_tolerance_auto_plan(shape):
    a, sa, b, sb = realistic_operands(*shape)
    c = blockfp8.gemm(a, sa, b, sb)
    assert_close(c, oracle_gemm(a, sa, b, sb))
    assert torch.equal(c, blockfp8.gemm(a, sa, b, sb))  # same plan, same bits


@pytest.mark.parametrize("config", CONFIGS)
def test_configs_agree_bitwise(config):
    # Every configuration computes each output the same way (four K = 32
    # MMAs per block from zero, one fmaf promotion per block, in order).
    _tokens(config, 100)
    a, sa, b, sb = realistic_operands(100, 520, 1040, seed=21)
    assert torch.equal(blockfp8.gemm(a, sa, b, sb, config=config, split_k=1),
                       blockfp8.gemm(a, sa, b, sb, config=0, split_k=1))


@pytest.mark.parametrize("col_major", [True, False])
def test_both_activation_scale_layouts(col_major):
    a, sa, b, sb = realistic_operands(70, 256, 640, col_major=col_major)
    c = blockfp8.gemm(a, sa, b, sb)
    c2 = blockfp8.gemm(a, sa.contiguous() if col_major else sa.t().contiguous().t(), b, sb)
    assert torch.equal(c, c2)
    assert_close(c, oracle_gemm(a, sa, b, sb))


@pytest.mark.parametrize("config, splits", [(0, 1), (0, 4), (1, 1), (1, 8), (2, 5)])
def test_bitwise_deterministic(config, splits):
    a, sa, b, sb = realistic_operands(48, 1024, 4096, seed=3)
    outs = [blockfp8.gemm(a, sa, b, sb, config=config, split_k=splits) for _ in range(5)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    assert_close(outs[0], oracle_gemm(a, sa, b, sb))


def test_split_k_inside_cuda_graph():
    a, sa, b, sb = realistic_operands(4, 4096, 4096, seed=4)
    eager = blockfp8.gemm(a, sa, b, sb, config=1, split_k=8)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        blockfp8.gemm(a, sa, b, sb, config=1, split_k=8)  # warm-up allocations
        with torch.cuda.graph(graph, stream=s):
            out = blockfp8.gemm(a, sa, b, sb, config=1, split_k=8)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)


def test_cancellation_across_blocks():
    # Block 1 is block 0 negated: the exact result is zero.
    a, sa, b, sb = realistic_operands(40, 256, 128, seed=5)
    a2, sa2 = torch.cat([a, a], dim=1), torch.cat([sa, sa], dim=1)
    b2 = torch.cat([b, (-b.float()).to(FP8)], dim=1)
    sb2 = torch.cat([sb, sb], dim=1)
    big = oracle_gemm(a, sa, b, sb, absolute=True)
    for config in CONFIGS:
        if (token_limit(blockfp8.configs()[config]) or 40) < 40:
            continue
        c = blockfp8.gemm(a2, sa2, b2, sb2, config=config)
        ref = oracle_gemm(a2, sa2, b2, sb2)
        err = np.abs(c.double().cpu().numpy() - ref)
        assert np.all(err <= 2.0 ** -8 * np.abs(ref) + 2.0 ** -12 * big + 1e-30), config


def test_cancellation_leaves_small_residual():
    a, sa, b, sb = realistic_operands(24, 384, 128, seed=6)
    a3 = torch.cat([a, a, a], dim=1)
    b3 = torch.cat([b, (-b.float()).to(FP8), b], dim=1)
    sa3 = torch.cat([sa, sa, sa * 2.0 ** -12], dim=1)
    sb3 = torch.cat([sb, sb, sb], dim=1)
    c = blockfp8.gemm(a3, sa3, b3, sb3)
    ref = oracle_gemm(a3, sa3, b3, sb3)
    big = oracle_gemm(a, sa, b, sb, absolute=True)
    err = np.abs(c.double().cpu().numpy() - ref)
    assert np.all(err <= 2.0 ** -8 * np.abs(ref) + 2.0 ** -13 * big)


@pytest.mark.parametrize("log2_scale", [-60, -20, 20, 50])
def test_extreme_scales(log2_scale):
    a, sa, b, sb = realistic_operands(17, 256, 512, seed=7)
    sa = sa * 2.0 ** log2_scale
    sb = sb * 2.0 ** (-log2_scale // 2)
    assert_close(blockfp8.gemm(a, sa, b, sb), oracle_gemm(a, sa, b, sb))


def test_extreme_fp8_values():
    g = torch.Generator().manual_seed(8)
    m, n, k = 32, 128, 512
    choices = torch.tensor([448.0, -448.0, 2.0 ** -9, -(2.0 ** -9), 2.0 ** -6, 0.0])
    a = choices[torch.randint(0, 6, (m, k), generator=g)].to(FP8).to(DEV)
    b = choices[torch.randint(0, 6, (n, k), generator=g)].to(FP8).to(DEV)
    sa = torch.full((m, 4), 2.0 ** -10, device=DEV)
    sb = torch.full((1, 4), 2.0 ** -8, device=DEV)
    assert_close(blockfp8.gemm(a, sa, b, sb), oracle_gemm(a, sa, b, sb))


def test_outlier_channel_and_zero_rows():
    g = torch.Generator().manual_seed(9)
    x = torch.randn(20, 1024, generator=g)
    x[:, 77] *= 300.0
    x[3] = 0.0
    a, sa = O.quantize_activations(x.numpy())
    b, sb = O.quantize_weights((torch.randn(512, 1024, generator=g) * 0.02).numpy())
    a_t, b_t = torch.from_numpy(a).view(FP8).to(DEV), torch.from_numpy(b).view(FP8).to(DEV)
    sa_t, sb_t = torch.from_numpy(np.ascontiguousarray(sa)).to(DEV), torch.from_numpy(sb).to(DEV)
    c = blockfp8.gemm(a_t, sa_t, b_t, sb_t)
    assert torch.all(c[3] == 0)
    assert_close(c, O.reference_gemm(a, sa, b, sb))


def test_m_zero_returns_empty():
    a, sa, b, sb = realistic_operands(1, 256, 256)
    c = blockfp8.gemm(a[:0], sa[:0], b, sb)
    assert c.shape == (0, 256) and c.dtype == torch.bfloat16


def test_op_rejects_bad_shapes_itself():
    a, sa, b, sb = realistic_operands(4, 256, 256)
    with pytest.raises(RuntimeError, match="b_scales"):
        torch.ops.blockfp8.gemm(a, sa, b, sb[:1], -1, 0)


# ---- the quantizer ------------------------------------------------------------

@pytest.mark.parametrize("ties", [False, True])
@pytest.mark.parametrize("shape", [(1, 128), (7, 272), (33, 4096), (300, 1040)])
def test_quantize_cuda_equals_oracle(shape, ties):
    x = bf16_activations(*shape, seed=15, ties=ties)
    x[0, :16] = 0.0
    xd = x.to(DEV)
    for eps in (1e-10, 1e-2):
        q, s = blockfp8.quantize_cuda(xd, eps=eps)
        q2, s2 = oracle_quant(x, eps=eps)
        assert s.stride() == (1, shape[0])
        assert np.array_equal(codes(q), q2)
        assert np.array_equal(f32(s).view(np.uint32), s2.view(np.uint32))


def test_quantize_cuda_special_groups():
    x = bf16_activations(20, 1024, seed=12)
    x[:, 77] *= 300.0
    x[3] = 0.0
    x[5, 128:256] = 1e-38  # below eps * 448: the scale is floored at eps / 448
    for eps in (1e-10, 1e-4):
        q, s = blockfp8.quantize_cuda(x.to(DEV), eps=eps)
        q2, s2 = oracle_quant(x, eps=eps)
        assert np.array_equal(codes(q), q2) and np.array_equal(f32(s), s2)


# ---- fused activation quantization (gemm_bf16) ----------------------------------

FUSED = list(range(len(blockfp8.fused_configs()))) if blockfp8.native_available() else [0]


def _weights(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    b, sb = O.quantize_weights((torch.randn(n, k, generator=g) * 0.02).numpy())
    return torch.from_numpy(b).view(FP8).to(DEV), torch.from_numpy(sb).to(DEV)


def _quantized(x: torch.Tensor, eps=1e-10):
    q, s = oracle_quant(x, eps=eps)
    return (torch.from_numpy(q).view(FP8).to(DEV),
            torch.from_numpy(np.ascontiguousarray(s.T)).t().to(DEV))


@pytest.mark.parametrize("config", FUSED)
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("ties", [False, True])
def test_fused_equals_quantize_then_gemm(config, shape, ties):
    m, n, k = shape
    _tokens(config, m)
    x = bf16_activations(m, k, seed=sum(shape) % 1000, ties=ties)
    b, sb = _weights(n, k, seed=1)
    a, sa = _quantized(x)
    expect = blockfp8.gemm(a, sa, b, sb, config=0, split_k=1)
    c = blockfp8.gemm_bf16(x.to(DEV), b, sb, config=config, split_k=1)
    assert torch.equal(c, expect)


@pytest.mark.parametrize("config", FUSED)
@pytest.mark.parametrize("splits", [2, 3, 7])
def test_fused_split_k(config, splits):
    _tokens(config, 37)
    x = bf16_activations(37, 2048 + 16, seed=splits, ties=True)
    b, sb = _weights(392, 2048 + 16, seed=2)
    a, sa = _quantized(x)
    expect = blockfp8.gemm(a, sa, b, sb, config=0, split_k=splits)
    assert torch.equal(blockfp8.gemm_bf16(x.to(DEV), b, sb, config=config, split_k=splits), expect)


def test_fused_zero_rows_outliers_and_eps():
    x = bf16_activations(20, 1024, seed=12)
    x[:, 77] *= 300.0
    x[3] = 0.0
    x[5, 128:256] = 1e-38
    b, sb = _weights(512, 1024, seed=4)
    for eps in (1e-10, 1e-4):
        a, sa = _quantized(x, eps=eps)
        for config in FUSED:
            if (token_limit(blockfp8.configs()[config]) or 20) < 20:
                continue  # 20 tokens: more than a 16-token streaming tile holds
            c = blockfp8.gemm_bf16(x.to(DEV), b, sb, eps=eps, config=config, split_k=1)
            assert torch.equal(c, blockfp8.gemm(a, sa, b, sb, config=0, split_k=1))
            assert torch.all(c[3] == 0)


@pytest.mark.parametrize("m", [1, 4, 16, 64, 256])
def test_fused_auto_plan_and_linear(m):
    x = bf16_activations(m, 4096, seed=m)
    b, sb = _weights(6144, 4096, seed=5)
    a, sa = _quantized(x)
    xd = x.to(DEV)
    assert_close(blockfp8.gemm_bf16(xd, b, sb), oracle_gemm(a, sa, b, sb))
    expect = blockfp8.gemm_bf16(xd, b, sb) if blockfp8.prefers_fused(m, 6144, 4096) else \
        blockfp8.gemm(a, sa, b, sb)
    assert torch.equal(blockfp8.linear(xd, b, sb), expect)
    assert blockfp8.linear(xd[:0], b, sb).shape == (0, 6144)


def test_fused_inside_cuda_graph():
    x = bf16_activations(4, 4096, seed=13).to(DEV)
    b, sb = _weights(4096, 4096, seed=6)
    eager = blockfp8.gemm_bf16(x, b, sb, config=0, split_k=8)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        blockfp8.gemm_bf16(x, b, sb, config=0, split_k=8)
        with torch.cuda.graph(graph, stream=s):
            out = blockfp8.gemm_bf16(x, b, sb, config=0, split_k=8)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)


def test_fused_rejects_bad_input():
    b, sb = _weights(256, 256, seed=7)
    with pytest.raises(ValueError):
        blockfp8.gemm_bf16(torch.zeros(2, 256, device=DEV), b, sb)  # float32
    with pytest.raises(ValueError):
        blockfp8.gemm_bf16(torch.zeros(2, 512, device=DEV, dtype=torch.bfloat16)[:, ::2], b, sb)
    with pytest.raises(RuntimeError, match="b_scales"):
        torch.ops.blockfp8.gemm_bf16(torch.zeros(2, 256, device=DEV, dtype=torch.bfloat16),
                                     b, sb[:, :1], -1, 0, 1e-10)


def test_ops_trace_under_torch_compile():
    x = bf16_activations(8, 256, seed=14).to(DEV)
    b, sb = _weights(256, 256, seed=8)
    a, sa = _quantized(x.cpu())

    def f(x, a, sa):
        q, s = torch.ops.blockfp8.quantize(x, 1e-10)
        return torch.ops.blockfp8.gemm_bf16(x, b, sb, -1, 0, 1e-10) + \
            torch.ops.blockfp8.gemm(a, sa, b, sb, -1, 0) + torch.ops.blockfp8.linear(x, b, sb) + \
            torch.ops.blockfp8.gemm(q, s, b, sb, -1, 0)

    out = torch.compile(f, fullgraph=True)(x, a, sa)
    assert torch.equal(out, f(x, a, sa))


# ---- weight-streaming (decode) configurations -------------------------------------

@pytest.mark.parametrize("config", STREAM)
@pytest.mark.parametrize("m, n, k, splits", [(1, 6144, 4096, -148), (16, 4096, 12288, -148), (7, 520, 1040, -45),
                                             (3, 1000, 1040, -1000), (16, 24576, 4096, -148), (5, 264, 272, 1),
                                             (2, 392, 2064, 3), (13, 128, 128, -148)])
def test_stream_exact_integer(config, m, n, k, splits):
    """Exact-integer operands through every token tile, split count and
    stream-K grid (tiles cut across CTAs, ragged K and N tails)."""
    a, sa, b, sb = integer_operands(m, n, k, seed=m + n + (splits % 13))
    c = blockfp8.gemm(a, sa, b, sb, config=config, split_k=splits)
    assert_exact(c, oracle_gemm(a, sa, b, sb))


@pytest.mark.parametrize("config", STREAM)
def test_stream_one_split_agrees_bitwise_with_the_tile_kernels(config):
    """One split: every tile's K blocks in order in one CTA, the same
    promotion as every other configuration, so the same bits."""
    a, sa, b, sb = realistic_operands(9, 520, 1040, seed=21)
    assert torch.equal(blockfp8.gemm(a, sa, b, sb, config=config, split_k=1),
                       blockfp8.gemm(a, sa, b, sb, config=0, split_k=1))


@pytest.mark.parametrize("config", STREAM)
@pytest.mark.parametrize("m", [1, 4, 16])
def test_stream_fused_modes_bitwise_and_deterministic(config, m):
    """bf16 in: the quantization kernel + streaming GEMM (mode 1) and the
    streaming GEMM quantizing in its own warps (mode 2) both give
    gemm(quantize(x))'s bits, call after call, within the tolerance of the
    oracle."""
    from blockfp8_b200 import capi
    x = bf16_activations(m, 4096, seed=3 + m, ties=True).to(DEV)
    b, sb = _weights(6144, 4096, seed=1)
    q, s = capi.quantize(x)
    expect = capi.gemm(q, s, b, sb, config=config, splits=-148)
    for mode in (1, 2):
        for _ in range(2):
            assert torch.equal(capi.gemm(x, None, b, sb, config=config, splits=-148, fused=mode), expect), mode
    assert_close(expect, oracle_gemm(q, s, b, sb))
    from blockfp8_b200 import _native
    assert _native.device_status(reset=True) == 0


@pytest.mark.parametrize("config", STREAM)
def test_stream_refuses_more_tokens_than_its_tile(config):
    lim = token_limit(blockfp8.configs()[config])
    a, sa, b, sb = realistic_operands(lim + 1, 256, 256, seed=2)
    with pytest.raises(RuntimeError, match="tokens"):
        blockfp8.gemm(a, sa, b, sb, config=config, split_k=-148)
