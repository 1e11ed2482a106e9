"""Multi-rank host logic on CPU (gloo, world size 2) and on 2 GPUs (NCCL).

CPU ranks run the column-sharded and row-sharded layer with the CPU oracle
standing in for the GPU GEMM (test-only) and check that the shards
reassemble into the unsharded result, that every rank's quantized
activations are identical, and that a rank that dies is noticed by the
others through a short process-group timeout instead of a hang.  The 2-GPU
tests run the real kernels over NCCL.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from blockfp8_b200 import sharding

FP8 = torch.float8_e4m3fn


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, backend, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def test_block_slices_cover_everything_in_whole_blocks():
    for extent in (128, 136, 4096, 24576, 1000, 6144):
        for world in (1, 2, 4, 8):
            if -(-extent // 128) < world:
                with pytest.raises(ValueError):
                    sharding.block_slices(extent, world, 0)
                continue
            cuts = [sharding.block_slices(extent, world, r) for r in range(world)]
            assert cuts[0][0] == 0 and cuts[-1][1] == extent
            for (lo, hi), (lo2, _) in zip(cuts, cuts[1:]):
                assert hi == lo2 and lo % 128 == 0 and hi % 128 == 0
            widths = [hi - lo for lo, hi in cuts]
            assert max(widths) - min(widths) <= 128 + extent % 128
    assert [sharding.block_slices(24576, 8, r) for r in (0, 7)] == [(0, 3072), (21504, 24576)]


def _column_worker(rank, world, port, out):
    from oracle import oracle as O
    _init(rank, world, port, "gloo")
    try:
        g = torch.Generator().manual_seed(0)
        m, n, k = 9, 640, 384
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        w = torch.randn(n, k, generator=g) * 0.02
        b_np, sb_np = O.quantize_weights(w.numpy())
        b, sb = torch.from_numpy(b_np).view(FP8), torch.from_numpy(sb_np)
        b_loc, sb_loc, (lo, hi) = sharding.shard_columns(b, sb, world, rank)
        # the slice's block scales are the scales of the sliced weights
        _, sb_check = O.quantize_weights(w[lo:hi].numpy())
        assert np.array_equal(sb_loc.numpy(), sb_check)
        a_np, sa_np = O.quantize_activations(x.view(torch.int16).numpy().view(np.uint16))
        # every rank quantized the replicated x identically
        digest = torch.tensor([int(a_np.astype(np.int64).sum()), int(sa_np.view(np.int32).astype(np.int64).sum())])
        digests = [torch.zeros_like(digest) for _ in range(world)]
        dist.all_gather(digests, digest)
        assert all(torch.equal(d, digests[0]) for d in digests)
        y_loc = torch.from_numpy(O.reference_gemm(a_np, sa_np, b_loc.view(torch.uint8).numpy(), sb_loc.numpy()))
        widths = [h - l for l, h in (sharding.block_slices(n, world, r) for r in range(world))]
        y = sharding.gather_columns(y_loc, widths)
        if rank == 0:
            full = O.reference_gemm(a_np, sa_np, b_np, sb_np)
            out["column"] = bool(np.array_equal(y.numpy(), full))
    finally:
        dist.destroy_process_group()


def _row_worker(rank, world, port, out):
    from oracle import oracle as O
    _init(rank, world, port, "gloo")
    try:
        g = torch.Generator().manual_seed(1)
        m, n, k = 5, 256, 1024
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        w = torch.randn(n, k, generator=g) * 0.02
        b_np, sb_np = O.quantize_weights(w.numpy())
        b, sb = torch.from_numpy(b_np).view(FP8), torch.from_numpy(sb_np)
        x_loc, b_loc, sb_loc, (lo, hi) = sharding.shard_rows(x, b, sb, world, rank)
        a_np, sa_np = O.quantize_activations(x_loc.contiguous().view(torch.int16).numpy().view(np.uint16))
        # K-slice quantization groups are the full quantization's groups
        a_full, sa_full = O.quantize_activations(x.view(torch.int16).numpy().view(np.uint16))
        assert np.array_equal(a_np, a_full[:, lo:hi]) and np.array_equal(sa_np, sa_full[:, lo // 128:hi // 128])
        y = torch.from_numpy(O.reference_gemm(a_np, sa_np, b_loc.contiguous().view(torch.uint8).numpy(),
                                              sb_loc.contiguous().numpy()))
        dist.all_reduce(y)
        if rank == 0:
            full = O.reference_gemm(a_full, sa_full, b_np, sb_np)
            out["row"] = float(np.abs(y.numpy() - full).max() / np.abs(full).max())
    finally:
        dist.destroy_process_group()


def _run(worker, world=2):
    port = _free_port()
    # spawn, not fork: the test process may already hold a CUDA context
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.spawn(worker, args=(world, port, out), nprocs=world, join=True)
        return dict(out)


def test_column_sharded_layer_on_two_gloo_ranks():
    assert _run(_column_worker)["column"] is True


def test_row_sharded_layer_all_reduce_on_two_gloo_ranks():
    assert _run(_row_worker)["row"] < 1e-12  # float64 partial sums: only rounding of the sum


def _dying_worker(rank, world, port, out):
    _init(rank, world, port, "gloo", timeout_s=3)
    if rank == 1:
        os._exit(0)  # leaves between steps, without a goodbye
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        out["noticed"] = False
    except Exception as e:  # the short process-group timeout ends the collective
        out["noticed"] = True
        out["error"] = type(e).__name__


def test_a_dead_rank_is_noticed_by_a_timeout_not_a_hang():
    port = _free_port()
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank hung"
        assert out.get("noticed") is True


# ---- two GPUs, NCCL ---------------------------------------------------------------

def _gpu_worker(rank, world, port, out):
    import blockfp8_b200 as bf
    from oracle import oracle as O
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl", timeout_s=120)
    try:
        dev = torch.device("cuda", rank)
        g = torch.Generator().manual_seed(2)
        m, n, k = 64, 2048, 4096
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        w = torch.randn(n, k, generator=g) * 0.02
        b_np, sb_np = O.quantize_weights(w.numpy())
        b, sb = torch.from_numpy(b_np).view(FP8), torch.from_numpy(sb_np)
        # column-parallel: exact gather of the single-GPU kernel's columns
        b_loc, sb_loc, (lo, hi) = sharding.shard_columns(b, sb, world, rank)
        y_loc = bf.linear(x.to(dev), b_loc.to(dev), sb_loc.to(dev))
        widths = [h - l for l, h in (sharding.block_slices(n, world, r) for r in range(world))]
        y = sharding.gather_columns(y_loc, widths)
        y_single = bf.linear(x.to(dev), b.to(dev), sb.to(dev))
        # row-parallel: NCCL sum of bf16 partials, within the parity tolerance
        x_loc, bk, sbk, _ = sharding.shard_rows(x, b, sb, world, rank)
        y_row = sharding.row_parallel_linear(x_loc.to(dev), bk.to(dev), sbk.to(dev))
        if rank == 0:
            a_np, sa_np = O.quantize_activations(x.view(torch.int16).numpy().view(np.uint16))
            ref = O.reference_gemm(a_np, sa_np, b_np, sb_np)
            tol = 1e-2 * np.abs(ref) + 1e-2 * np.abs(ref).max()
            out["column_exact"] = bool(torch.equal(y, y_single))
            out["row_ok"] = bool(np.all(np.abs(y_row.double().cpu().numpy() - ref) <= tol))
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_column_and_row_parallel_on_two_gpus():
    out = _run(_gpu_worker)
    assert out["column_exact"] and out["row_ok"], out
