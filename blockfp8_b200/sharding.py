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
and 128x128 weight blocks are the same as unsharded).  Two ways to sum the
ranks' [M, N] partials:
- row_parallel_linear: linear, then an NCCL all-reduce of the bf16 outputs
  (what vLLM's RowParallelLinear does around the block-FP8 GEMM);
- RowParallelGroup.linear: the all-reduce inside the GEMM kernel over
  NVLink peer memory (bfp8_launch_gemm_tp): fp32 tile sums meet at one
  rank, are added in rank order and rounded once, and every rank receives
  the bf16 tiles as they finish; no second kernel and no bf16 rounding of
  the partials.
"""

import ctypes

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


class _DeviceBuffer:
    """A raw device allocation seen by torch.as_tensor (CUDA array interface)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class RowParallelGroup:
    """Row-parallel block-FP8 linear layers of one process group whose
    all-reduce runs inside the GEMM (bfp8_launch_gemm_tp).

    Every rank allocates its partial, counter and output buffers once
    (sized for up to max_m rows of an N-wide output), exports them as CUDA
    IPC handles, and maps every other rank's (one all_gather_object at
    construction).  All ranks must then make the same linear() calls in the
    same order, each with its own K slice (block_slices(k, world, rank)) of x
    and of the weight; every rank runs the same plan (tile ids must agree),
    chosen for the widest slice.  The returned [M, N] tensor lives in the
    group's output buffer: the same bits on every rank, valid until the
    group's next call (clone it to keep it).  If a rank stops calling, the
    others' kernels give up their bounded wait after about 2 s and
    _native.device_status() reports it; the group must then be rebuilt.
    """

    def __init__(self, max_m: int, n: int, k: int, group=None, device=None):
        import torch.distributed as dist

        from . import _native, capi

        self._lib = _native.capi()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= _native.TP_MAX_RANKS:
            raise ValueError(f"row-parallel groups hold 1 to {_native.TP_MAX_RANKS} ranks, not {self.world}")
        if n % 8 or max_m < 1:
            raise ValueError("n must be a multiple of 8 and max_m positive")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.max_m, self.n, self.k = max_m, n, k
        self.k_lo, self.k_hi = block_slices(k, self.world, self.rank, GROUP_K)
        self.k_plan = block_slices(k, self.world, 0, GROUP_K)[1]  # the widest slice
        # the largest partial buffer and tile count any plan can ask for at max_m rows
        probe = _native.GemmProblem(M=max_m, N=n, K=128)
        part, tiles = 16, 1
        for cfg in range(self._lib.bfp8_num_configs()):
            plan = _native.Plan(cfg, 1, 0)
            if self._lib.bfp8_tp_tiles(ctypes.byref(probe), plan) < 0:
                continue  # no row-parallel variant (the weight-streaming configurations)
            part = max(part, capi.tp_partial_bytes(probe, plan, self.world))
            tiles = max(tiles, capi.tp_tiles(probe, plan))
        sizes = (part, 8 * (2 + tiles), 2 * max_m * n)
        self._own, handles = [], []
        with torch.cuda.device(self.device):
            for nbytes in sizes:
                ptr, h = ctypes.c_void_p(), ctypes.create_string_buffer(_native.IPC_HANDLE_BYTES)
                _native.check(self._lib.bfp8_tp_alloc(nbytes, ctypes.byref(ptr), h))
                self._own.append(ptr.value)
                handles.append(h.raw)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, handles, group=group)
        self._mapped = []
        self.partials, self.counters, self.outs = [], [], []
        with torch.cuda.device(self.device):
            for q, hs in enumerate(everyone):
                ptrs = []
                for i, h in enumerate(hs):
                    if q == self.rank:
                        ptrs.append(self._own[i])
                        continue
                    ptr = ctypes.c_void_p()
                    _native.check(self._lib.bfp8_tp_open(h, ctypes.byref(ptr)))
                    self._mapped.append(ptr.value)
                    ptrs.append(ptr.value)
                self.partials.append(ptrs[0])
                self.counters.append(ptrs[1])
                self.outs.append(ptrs[2])
        self._group = group
        self.broken = False

    def linear(self, x: torch.Tensor, b_q: torch.Tensor, b_scales: torch.Tensor, check: bool = False) -> torch.Tensor:
        """sum over ranks of x_r @ W_r^T for this rank's x_r [M, K_r] (bf16) and
        block-FP8 W_r [N, K_r]; [M, N] bf16, identical on every rank.

        check=True synchronises after the launch and raises RuntimeError if
        a bounded wait of the kernel gave up (another rank stalled or never
        launched): the output is then incomplete.  Once a wait has given up
        the group's counters are inconsistent, so every later call raises
        until the group is rebuilt (a check=False call cannot know; read
        blockfp8_b200._native.device_status() to find out)."""
        from . import _native, capi
        from .layout import FP8_DTYPE

        if self.broken:
            raise RuntimeError("this row-parallel group saw a wait give up; close it and build a new one")

        if x.dtype != torch.bfloat16 or x.dim() != 2 or b_q.dtype != FP8_DTYPE or b_q.dim() != 2:
            raise ValueError("x must be 2-D bf16 and b_q 2-D float8_e4m3fn")
        m, n = x.shape[0], b_q.shape[0]
        if n != self.n or m > self.max_m:
            raise ValueError(f"the group serves N = {self.n} and up to {self.max_m} rows, got [{m}, {n}]")
        if x.shape[1] != self.k_hi - self.k_lo or b_q.shape[1] != x.shape[1]:
            raise ValueError(f"rank {self.rank} holds K columns [{self.k_lo}, {self.k_hi}), got x {tuple(x.shape)}, "
                             f"b_q {tuple(b_q.shape)}")
        out = torch.as_tensor(_DeviceBuffer(self.outs[self.rank], (self.max_m, n), "<i2"),
                              device=self.device).view(torch.bfloat16)[:m]
        if m == 0:
            return out
        x = x.contiguous()
        fused = bool(self._lib.bfp8_prefers_fused(m, n, self.k_plan))
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        plan = self._lib.bfp8_choose_tp_plan(m, n, self.k_plan, sms, int(fused))
        if fused:
            p = capi.problem(x, None, b_q, b_scales, out)
        else:
            q, s = capi.quantize(x)
            p = capi.problem(q, s, b_q, b_scales, out)
        ws, cnt = capi.scratch(p, plan, self.device)
        tp = _native.TpGroup(world=self.world, rank=self.rank, wait=1)
        for qr in range(self.world):
            tp.partials[qr], tp.counters[qr], tp.out[qr] = self.partials[qr], self.counters[qr], self.outs[qr]
        capi.launch_gemm_tp(p, plan, tp, ws, cnt)
        if check:
            status = _native.device_status(reset=False)
            if status:
                self.broken = True
                raise RuntimeError(f"a bounded wait of the row-parallel kernel gave up (status {status:#x}); "
                                   "the output is incomplete and the group must be rebuilt")
        return out

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank's
        last call has finished: a barrier on the group first)."""
        import torch.distributed as dist

        if not self._own:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self._group)
        with torch.cuda.device(self.device):
            for ptr in self._mapped:
                self._lib.bfp8_tp_close(ctypes.c_void_p(ptr))
            for ptr in self._own:
                self._lib.bfp8_tp_free(ctypes.c_void_p(ptr))
        self._own, self._mapped = [], []
