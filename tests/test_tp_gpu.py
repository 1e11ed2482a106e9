"""Row-parallel GEMM with its all-reduce inside the kernel (bfp8_launch_gemm_tp).

On one GPU the ranks of a group run one after another, each with its own
partial, counter and output buffers and wait = 0 (no kernel waits for
another launch): every rank but the last only hands its tiles over, the
last sums them and delivers every rank's output.  That covers the whole
kernel path except the NVLink transport, which the two-GPU test covers.
Checks: exact-integer operands bit-exact against the oracle; realistic
operands within the parity tolerance of the unsharded product; every
rank's output identical; repeated calls (counter reset, delivery counts)
identical; world = 1 identical to the ordinary launch.
"""

import os

import numpy as np
import pytest
import torch

import blockfp8_b200 as bf
from blockfp8_b200 import _native, capi, sharding
from helpers import assert_close, assert_exact, integer_operands, oracle_gemm, realistic_operands

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU"),
]

DEV = "cuda"


def _names():
    return bf.configs() if bf.native_available() else []


def _rank_problem(a, sa, b, sb, out, lo, hi, fused):
    """This rank's problem: its K columns [lo, hi) of a (or bf16 x), sa, b, sb."""
    kb0, kb1 = lo // 128, -(-hi // 128)
    if fused:
        return capi.problem(a[:, lo:hi], None, b[:, lo:hi], sb[:, kb0:kb1], out)
    return capi.problem(a[:, lo:hi], sa[:, kb0:kb1], b[:, lo:hi], sb[:, kb0:kb1], out)


def emulate(world, a, sa, b, sb, plan, rounds=2, fused=False):
    """Run `world` ranks one after another; returns (outputs of every rank per
    round, counters of every rank after the last round, tiles per call)."""
    m, k = a.shape
    n = b.shape[0]
    slices = [sharding.block_slices(k, world, r, 128) for r in range(world)]
    probe = _native.GemmProblem(M=m, N=n, K=k)
    tiles = capi.tp_tiles(probe, plan)
    part_bytes = capi.tp_partial_bytes(probe, plan, world)
    partials = [torch.zeros(part_bytes // 4, dtype=torch.float32, device=DEV) for _ in range(world)]
    counters = [torch.zeros(2 + tiles, dtype=torch.int64, device=DEV) for _ in range(world)]
    outs = [torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    results = []
    for rnd in range(rounds):
        for r in range(world):
            p = _rank_problem(a, sa, b, sb, outs[r], *slices[r], fused)
            ws, cnt = capi.scratch(p, plan, a.device)
            tp = _native.TpGroup(world=world, rank=r, wait=1 if world == 1 else 0)
            for q in range(world):
                tp.partials[q] = partials[q].data_ptr()
                tp.counters[q] = counters[q].data_ptr()
                tp.out[q] = outs[q].data_ptr()
            capi.launch_gemm_tp(p, plan, tp, ws, cnt)
        torch.cuda.synchronize()
        assert _native.device_status(reset=True) == 0
        results.append([o.clone() for o in outs])
    return results, [c.cpu() for c in counters], tiles


def _check_group(results, counters, tiles, rounds):
    first = results[0][0]
    for outs in results:
        for o in outs:
            assert torch.equal(o.view(torch.int16), first.view(torch.int16)), "ranks or rounds differ"
    for c in counters:
        assert c[0].item() == rounds * tiles, "delivered-tile count"
        assert c[1].item() == rounds * tiles, "taken-tile count"
        assert torch.count_nonzero(c[2:]).item() == 0, "tile counters not reset"
    return first


PLANS = [("m128n256s4", 1), ("m128n128s6", 2), ("m128n64s8", 1), ("m256n256s6", 1),
         ("w128t16s10", 3), ("w128t32s10", -40), ("w128t64s8", 1)]


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("cfg, splits", PLANS)
def test_integer_operands_bit_exact(world, cfg, splits):
    """Exact partial sums: every rank's output equals the oracle's rounding
    of the exact product, for every configuration, local split-K and
    stream-K included."""
    m, n, k = (5, 392, 1152) if cfg.startswith("w") else (300, 520, 1152)
    a, sa, b, sb = integer_operands(m, n, k, seed=world)
    plan = _native.Plan(_names().index(cfg), splits, 0)
    results, counters, tiles = emulate(world, a, sa, b, sb, plan)
    out = _check_group(results, counters, tiles, 2)
    assert_exact(out, oracle_gemm(a, sa, b, sb))


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("shape", [(16, 4096, 4096), (256, 4096, 3072), (33, 1024, 12288)])
def test_realistic_operands_match_the_unsharded_product(world, shape):
    m, n, k = shape
    a, sa, b, sb = realistic_operands(m, n, k, seed=m)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    plan = _native.capi().bfp8_choose_tp_plan(m, n, sharding.block_slices(k, world, 0, 128)[1], sms, 0)
    results, counters, tiles = emulate(world, a, sa, b, sb, plan)
    out = _check_group(results, counters, tiles, 2)
    ref = oracle_gemm(a, sa, b, sb)
    assert_close(out, ref)
    ref_abs = oracle_gemm(a, sa, b, sb, absolute=True)
    err = (out.double().cpu() - torch.from_numpy(ref)).abs()
    assert torch.all(err <= bf.error_bound(torch.from_numpy(ref), torch.from_numpy(ref_abs), k))


@pytest.mark.parametrize("mode", [1, 2])
def test_fused_quantization_plans(mode):
    """bf16 activations in: each rank quantizes its own K slice (the groups
    are the same as unsharded, K slices being whole 128-column blocks)."""
    m, n, k, world = 24, 512, 1024, 2
    g = torch.Generator().manual_seed(3)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    b, sb = bf.quantize_weights(torch.randn(n, k, generator=g).to(DEV) * 0.02)
    q, s = bf.quantize_cuda(x)
    plan = _native.Plan(_names().index("w128t32s10"), 2, mode)
    results, counters, tiles = emulate(world, x, None, b, sb, plan, fused=True)
    out = _check_group(results, counters, tiles, 2)
    assert_close(out, oracle_gemm(q, s, b, sb))


def test_world_of_one_equals_the_ordinary_launch():
    m, n, k = 200, 768, 2048
    a, sa, b, sb = realistic_operands(m, n, k, seed=9)
    for cfg, splits in PLANS:
        plan = _native.Plan(_names().index(cfg), splits, 0)
        results, counters, tiles = emulate(1, a, sa, b, sb, plan, rounds=3)
        out = _check_group(results, counters, tiles, 3)
        c = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
        p = capi.problem(a, sa, b, sb, c)
        ws, cnt = capi.scratch(p, plan, a.device)
        capi.launch_gemm(p, plan, ws, cnt)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), c.view(torch.int16)), cfg


def test_argument_checks():
    m, n, k = 16, 256, 512
    a, sa, b, sb = realistic_operands(m, n, k, seed=1)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    other = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    p = capi.problem(a, sa, b, sb, out)
    plan = _native.Plan(0, 1, 0)
    cnt = torch.zeros(64, dtype=torch.int64, device=DEV)
    part = torch.zeros(1 << 20, dtype=torch.float32, device=DEV)
    tp = _native.TpGroup(world=2, rank=0, wait=0)
    tp.partials[0] = tp.partials[1] = part.data_ptr()
    tp.counters[0] = tp.counters[1] = cnt.data_ptr()
    tp.out[0], tp.out[1] = other.data_ptr(), out.data_ptr()
    with pytest.raises(RuntimeError, match="out\\[rank\\]"):
        capi.launch_gemm_tp(p, plan, tp)
    tp.out[1] = 0
    tp.out[0] = out.data_ptr()
    with pytest.raises(RuntimeError, match="null tp buffer"):
        capi.launch_gemm_tp(p, plan, tp)


def _two_gpu_worker(rank, world, port, results):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        n, k = 4096, 4096
        grp = sharding.RowParallelGroup(max_m=512, n=n, k=k)
        g = torch.Generator().manual_seed(0)
        w = torch.randn(n, k, generator=g) * 0.02
        b, sb = bf.quantize_weights(w.cuda())
        lo, hi = grp.k_lo, grp.k_hi
        b_r, sb_r = b[:, lo:hi].contiguous(), sb[:, lo // 128:hi // 128].contiguous()
        out = {}
        for m in (1, 16, 300, 512, 16):  # shapes change between calls: delivery targets add up
            x = (torch.randn(m, k, generator=g) * 2).to(torch.bfloat16).cuda()
            y = grp.linear(x[:, lo:hi], b_r, sb_r).clone()
            y_nccl = sharding.row_parallel_linear(x[:, lo:hi], b_r, sb_r)
            full = bf.linear(x, b, sb)
            torch.cuda.synchronize()
            gathered = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(gathered, y)
            out[m] = (all(torch.equal(t.view(torch.int16), y.view(torch.int16)) for t in gathered),
                      float((y.float() - full.float()).abs().max()), float((y_nccl.float() - full.float()).abs().max()),
                      float(full.float().abs().max()))
        # The group keeps no per-call host state: a captured call replays.
        x = (torch.randn(16, k, generator=g) * 2).to(torch.bfloat16).cuda()
        xr = x[:, lo:hi].contiguous()
        eager = grp.linear(xr, b_r, sb_r).clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            grp.linear(xr, b_r, sb_r)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y_graph = grp.linear(xr, b_r, sb_r)
        replays_equal = True
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            replays_equal = replays_equal and torch.equal(y_graph.view(torch.int16), eager.view(torch.int16))
        del graph
        out["graph"] = replays_equal
        assert _native.device_status(reset=True) == 0
        grp.close()
        if rank == 0:
            results.update(out)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_over_nvlink():
    """Two processes, one GPU each: the fused row-parallel linear gives the
    same bits on both ranks, and agrees with the unsharded linear as closely
    as linear + NCCL all-reduce does."""
    import torch.multiprocessing as mp

    results = mp.Manager().dict()
    port = 29500 + os.getpid() % 1000
    mp.spawn(_two_gpu_worker, args=(2, port, results), nprocs=2, join=True)
    assert set(results.keys()) == {1, 16, 300, 512, "graph"}
    assert results.pop("graph"), "graph replays differ from the eager call"
    for m, (same, err, err_nccl, amax) in results.items():
        assert same, f"ranks differ at M={m}"
        assert err <= 1e-2 * amax, (m, err, amax)
        assert err <= err_nccl + 2 ** -8 * amax, (m, err, err_nccl)
