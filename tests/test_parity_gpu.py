"""Parity on the benchmark's own configurations and at vLLM's boundary (GPU).

- Configuration 1 of the benchmark (one qkv linear, M = 256, N = 6144,
  K = 4096, seeded N(0, 1) bf16 activations, N(0, 0.02) weights): the full
  output of blockfp8.linear against the CPU oracle, the quantized bytes and
  scales bit-exact.
- The prefill sweep's off-grid M (100, 384, 768, 3000) on the four Qwen3-8B
  linear shapes under the automatic plan: full outputs up to M = 768, the
  first and last 128 rows at M = 3000.
- vLLM feeds this path through its own quantizer,
  per_token_group_quant_fp8 (the reference pins its kernels to it bitwise,
  simon-jd/blockfp8 tests/test_gemm_gpu.py:323-335): the same bytes and
  scales from quantize_cuda, and linear / gemm_bf16 equal to gemm on vLLM's
  quantized activations.
- A bounded wait made to run out: the row-parallel kernel of rank 0 of a
  two-rank group, launched alone with wait = 1, gives up after its limit,
  records site 8 in the status word and returns (no GPU fault, the context
  stays usable).
"""

import time

import numpy as np
import pytest
import torch

import blockfp8
from blockfp8_b200 import _native, capi
from helpers import FP8, assert_close, bf16_activations, codes, f32, oracle_quant
from oracle import oracle as O

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

DEV = "cuda"
SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (24576, 4096), "down": (4096, 12288)}


def _benchmark_operands(m, n, k, seed=0):
    """The benchmark's data: x ~ N(0, 1) as bf16 and w ~ N(0, 0.02) from one
    CPU generator seeded `seed`, w quantized in 128 x 128 blocks (oracle)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = torch.randn(n, k, generator=g) * 0.02
    b, sb = O.quantize_weights(w.numpy())
    return x, b, sb, torch.from_numpy(b).view(FP8).to(DEV), torch.from_numpy(sb).to(DEV)


def test_config1_qkv_m256_full_output():
    x, b_np, sb_np, b, sb = _benchmark_operands(256, 6144, 4096, seed=0)
    xd = x.to(DEV)
    q, s = blockfp8.quantize_cuda(xd)
    a_np, sa_np = oracle_quant(x)
    assert np.array_equal(codes(q), a_np) and np.array_equal(f32(s), sa_np)
    y = blockfp8.linear(xd, b, sb)
    assert_close(y, O.reference_gemm(a_np, sa_np, b_np, sb_np))
    assert _native.device_status(reset=True) == 0


@pytest.mark.parametrize("layer", sorted(SHAPES))
@pytest.mark.parametrize("m", [100, 384, 768, 3000])
def test_off_grid_prefill_m_auto_plan(layer, m):
    n, k = SHAPES[layer]
    x, b_np, sb_np, b, sb = _benchmark_operands(m, n, k, seed=m)
    y = blockfp8.linear(x.to(DEV), b, sb)
    rows = np.arange(m) if m <= 768 else np.r_[0:128, m - 128:m]
    a_np, sa_np = oracle_quant(x[torch.from_numpy(rows)])
    ref = O.reference_gemm(a_np, sa_np, b_np, sb_np)
    assert_close(y[torch.from_numpy(rows).to(DEV)], ref)
    assert _native.device_status(reset=True) == 0


def _vllm_quant():
    try:
        from vllm.model_executor.layers.quantization.utils.fp8_utils import per_token_group_quant_fp8
    except Exception:
        return None
    return lambda x: per_token_group_quant_fp8(x, 128, column_major_scales=True, use_ue8m0=False)


@pytest.mark.skipif(_vllm_quant() is None, reason="vLLM not importable")
@pytest.mark.parametrize("ties", [False, True])
@pytest.mark.parametrize("m, n, k", [(1, 4096, 4096), (16, 6144, 4096), (64, 4096, 12288), (300, 1024, 4096)])
def test_quantizer_and_fused_paths_equal_vllms_quantizer(m, n, k, ties):
    x = bf16_activations(m, k, seed=11 + m, ties=ties).to(DEV)
    _, _, _, b, sb = _benchmark_operands(8, n, k, seed=3)
    q_v, s_v = _vllm_quant()(x)
    q, s = blockfp8.quantize_cuda(x)
    assert torch.equal(q.view(torch.uint8), q_v.view(torch.uint8)) and torch.equal(s, s_v.float())
    expect = blockfp8.gemm(q_v, s_v.float(), b, sb)
    assert torch.equal(blockfp8.linear(x, b, sb), expect)
    assert torch.equal(blockfp8.gemm_bf16(x, b, sb, config=0, split_k=1),
                       blockfp8.gemm(q_v, s_v.float(), b, sb, config=0, split_k=1))


def test_row_parallel_delivery_wait_gives_up_and_reports():
    """Rank 0 of two, alone: the other rank's tiles never arrive.  CTA 0's
    end-of-kernel wait for this rank's output gives up after its bounded
    limit (about 2 s), writes (0x5B << 56) | (8 << 32) | ... to the status
    word and the kernel returns; the next launch on the device works."""
    m, n, k, world = 16, 512, 1024, 2
    g = torch.Generator().manual_seed(4)
    a = torch.randint(-4, 5, (m, k), generator=g).float().to(FP8).to(DEV)
    sa = torch.ones(m, k // 128, device=DEV)
    b = torch.randint(-4, 5, (n, k), generator=g).float().to(FP8).to(DEV)
    sb = torch.ones(n // 128, k // 128, device=DEV)
    plan = _native.Plan(blockfp8.configs().index("w128t16s10"), 1, 0)
    probe = _native.GemmProblem(M=m, N=n, K=k // world)
    tiles = capi.tp_tiles(probe, plan)
    part_bytes = capi.tp_partial_bytes(probe, plan, world)
    partials = [torch.zeros(part_bytes // 4, dtype=torch.float32, device=DEV) for _ in range(world)]
    counters = [torch.zeros(2 + tiles, dtype=torch.int64, device=DEV) for _ in range(world)]
    outs = [torch.zeros(m, n, dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    assert _native.device_status(reset=True) == 0
    tp = _native.TpGroup(world=world, rank=0, wait=1)
    for r in range(world):
        tp.partials[r], tp.counters[r], tp.out[r] = (partials[r].data_ptr(), counters[r].data_ptr(),
                                                     outs[r].data_ptr())
    kb = k // world // 128
    p = capi.problem(a[:, : k // world], sa[:, :kb], b[:, : k // world], sb[:, :kb], outs[0])
    ws, cnt = capi.scratch(p, plan, a.device)
    t0 = time.perf_counter()
    capi.launch_gemm_tp(p, plan, tp, ws, cnt)
    status = _native.device_status(reset=True)  # synchronises
    elapsed = time.perf_counter() - t0
    assert status >> 56 == 0x5B and (status >> 32) & 0xFFFF == 8, hex(status)
    assert elapsed < 30, elapsed
    # the context is still usable
    c = blockfp8.gemm(a, sa, b, sb)
    torch.cuda.synchronize()
    assert _native.device_status(reset=True) == 0 and torch.isfinite(c.float()).all()
