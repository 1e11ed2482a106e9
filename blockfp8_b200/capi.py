"""ctypes binding of the C ABI (include/blockfp8_b200.h) for torch tensors.

The torch-free route into the kernels: every call goes straight to
libblockfp8_b200.so with raw device pointers, the way a non-PyTorch host
(or a test) would bind it.  Workspace and counters are the caller's.
"""

import ctypes

import torch

from . import _native
from ._native import GemmProblem, Plan, QuantProblem, check


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(stream=None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def problem(a, a_scales, b, b_scales, c, eps: float = 1e-10) -> GemmProblem:
    p = GemmProblem()
    p.a, p.lda = a.data_ptr(), a.stride(0)
    p.b, p.ldb = b.data_ptr(), b.stride(0)
    if a_scales is not None:
        p.sa, p.sa_m, p.sa_k = a_scales.data_ptr(), a_scales.stride(0), a_scales.stride(1)
    p.sb, p.sb_n, p.sb_k = b_scales.data_ptr(), b_scales.stride(0), b_scales.stride(1)
    p.c, p.ldc = c.data_ptr(), c.stride(0)
    p.M, p.N, p.K = a.shape[0], b.shape[0], b.shape[1]
    p.eps = eps
    return p


def choose_plan(m: int, n: int, k: int, num_sms: int, fused: bool = False) -> Plan:
    lib = _native.capi()
    return (lib.bfp8_choose_fused_plan if fused else lib.bfp8_choose_plan)(m, n, k, num_sms)


def scratch(p: GemmProblem, plan: Plan, device) -> tuple:
    """(workspace, counters) tensors sized for this plan (None where not needed)."""
    lib = _native.capi()
    nbytes = lib.bfp8_workspace_bytes(ctypes.byref(p), plan)
    check(nbytes if nbytes < 0 else 0)
    ncount = lib.bfp8_counters_needed(ctypes.byref(p), plan)
    check(ncount if ncount < 0 else 0)
    ws = torch.empty((nbytes + 3) // 4, dtype=torch.float32, device=device) if nbytes else None
    cnt = torch.zeros(ncount, dtype=torch.int32, device=device) if ncount else None
    return ws, cnt


def launch_gemm(p: GemmProblem, plan: Plan, workspace=None, counters=None, stream=None) -> None:
    check(_native.capi().bfp8_launch_gemm(ctypes.byref(p), plan, _ptr(workspace), _ptr(counters),
                                          _stream(stream)))


def gemm(a, a_scales, b, b_scales, config: int = -1, splits: int = 0, fused=False,
         eps: float = 1e-10, stream=None) -> torch.Tensor:
    """C = block-scaled A @ B^T through the C ABI alone (A bf16 when fused).

    fused: False (A is e4m3 with a_scales), True (bf16 A, the library's
    fused plan), or a bfp8_plan.fused mode (1: quantization kernel + GEMM,
    2: quantization inside the GEMM where the plan allows it)."""
    c = torch.empty(a.shape[0], b.shape[0], dtype=torch.bfloat16, device=a.device)
    p = problem(a, a_scales, b, b_scales, c, eps)
    sms = torch.cuda.get_device_properties(a.device).multi_processor_count
    plan = choose_plan(p.M, p.N, p.K, sms, bool(fused))
    if config >= 0:
        plan.config, plan.splits = config, splits if splits != 0 else 1
    elif splits != 0:
        plan.splits = splits  # < 0: stream-K over -splits CTAs
    if fused is not True and fused is not False:
        plan.fused = int(fused)
    ws, cnt = scratch(p, plan, a.device)
    launch_gemm(p, plan, ws, cnt, stream)
    return c


def quantize(x: torch.Tensor, eps: float = 1e-10, stream=None):
    """(q [M, K] e4m3, M-major scales) through the C ABI."""
    m, k = x.shape
    q = torch.empty(m, k, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty((k + 127) // 128, m, dtype=torch.float32, device=x.device).t()
    p = QuantProblem()
    p.x, p.ldx = x.data_ptr(), x.stride(0)
    p.q, p.ldq = q.data_ptr(), q.stride(0)
    p.s, p.s_m, p.s_k = s.data_ptr(), s.stride(0), s.stride(1)
    p.M, p.K, p.eps = m, k, eps
    check(_native.capi().bfp8_launch_quantize(ctypes.byref(p), _stream(stream)))
    return q, s


def launch_gemm_tp(p: GemmProblem, plan: Plan, tp: _native.TpGroup, workspace=None, counters=None,
                   stream=None) -> None:
    """bfp8_launch_gemm_tp: the GEMM of one rank of a row-parallel group, its
    all-reduce included (tp describes the group's buffers)."""
    check(_native.capi().bfp8_launch_gemm_tp(ctypes.byref(p), plan, _ptr(workspace), _ptr(counters),
                                             ctypes.byref(tp), _stream(stream)))


def tp_tiles(p: GemmProblem, plan: Plan) -> int:
    n = _native.capi().bfp8_tp_tiles(ctypes.byref(p), plan)
    check(n if n < 0 else 0)
    return n


def tp_partial_bytes(p: GemmProblem, plan: Plan, world: int) -> int:
    n = _native.capi().bfp8_tp_partial_bytes(ctypes.byref(p), plan, world)
    check(n if n < 0 else 0)
    return n
