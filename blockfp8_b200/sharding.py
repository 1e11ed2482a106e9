"""Tensor-parallel sharding of block-FP8 linear layers across GPUs.

Column-parallel (N split): each rank owns a contiguous slice of weight rows
whose bounds are multiples of 128, so every 128x128 weight-scale block stays
whole and the rank's slice of B_scales is a row slice of the full one.  The
activations are replicated and every rank quantizes them itself (the
quantizer is deterministic, so all ranks hold the same bits); there is no
collective on this path.  gather_columns reassembles the output, for
checking only.

Row-parallel (K split, for o/down in a tensor-parallel model): each rank
owns a contiguous K slice (multiples of 128, so the 1x128 activation groups
and 128x128 weight blocks are the same as unsharded), computes its partial
[M, N] with linear, and an all-reduce (NCCL over NVLink on GPUs) sums the
partials.
"""

import torch

from .layout import BLOCK_N, GROUP_K


def block_slices(extent: int, world: int, rank: int, block: int = 128) -> tuple[int, int]:
    """Contiguous [lo, hi) of `extent` for `rank`, cut at multiples of `block`;
    whole blocks are spread as evenly as possible (earlier ranks get the
    extra ones), and the ragged tail block goes to the last rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    blocks = -(-extent // block)
    if blocks < world:
        raise ValueError(f"{extent} is too small to give {world} ranks a {block}-wide slice each")
    base, extra = divmod(blocks, world)
    lo_b = rank * base + min(rank, extra)
    hi_b = lo_b + base + (1 if rank < extra else 0)
    return lo_b * block, min(hi_b * block, extent)


def shard_columns(b_q: torch.Tensor, b_scales: torch.Tensor, world: int, rank: int):
    """(b_q slice, b_scales slice, (lo, hi)) of the weight rows of `rank`."""
    lo, hi = block_slices(b_q.shape[0], world, rank, BLOCK_N)
    return b_q[lo:hi], b_scales[lo // BLOCK_N:-(-hi // BLOCK_N)], (lo, hi)


def shard_rows(x: torch.Tensor, b_q: torch.Tensor, b_scales: torch.Tensor, world: int, rank: int):
    """(x slice, b_q slice, b_scales slice, (lo, hi)) of the K range of `rank`."""
    lo, hi = block_slices(b_q.shape[1], world, rank, GROUP_K)
    return (x[:, lo:hi], b_q[:, lo:hi], b_scales[:, lo // GROUP_K:-(-hi // GROUP_K)], (lo, hi))


def gather_columns(y_local: torch.Tensor, widths: list[int], group=None) -> torch.Tensor:
    """All-gather column slices of widths[r] from every rank into [M, sum(widths)]."""
    import torch.distributed as dist
    m, wmax = y_local.shape[0], max(widths)
    padded = torch.zeros(m, wmax, dtype=y_local.dtype, device=y_local.device)
    padded[:, :y_local.shape[1]] = y_local
    parts = [torch.empty_like(padded) for _ in widths]
    dist.all_gather(parts, padded, group=group)  # equal sizes on every rank
    return torch.cat([p[:, :w] for p, w in zip(parts, widths)], dim=1)


def row_parallel_linear(x: torch.Tensor, b_q: torch.Tensor, b_scales: torch.Tensor, group=None):
    """linear on this rank's K slice, then a sum all-reduce of the [M, N] partials."""
    import torch.distributed as dist

    from .gemm import linear  # the submodule's function (the package re-exports a `gemm` function)
    y = linear(x.contiguous(), b_q.contiguous(), b_scales.contiguous())
    dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y
