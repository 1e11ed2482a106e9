"""Loading the native libraries: the C ABI (ctypes) and the torch op library.

libblockfp8_b200.so carries the kernels behind the C ABI declared in
include/blockfp8_b200.h; _C.so registers torch.ops.blockfp8.* on top of it.
Both are built in-tree by blockfp8_b200/build.py.  Nothing here falls back
to another implementation: when a library is missing, the functions that
need it raise.
"""

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
CAPI_LIB = os.path.join(HERE, "libblockfp8_b200.so")
OPS_LIB = os.path.join(HERE, "_C.so")

BFP8_OK = 0
BFP8_EINVAL = -1
BFP8_ECUDA = -2


class GemmProblem(ctypes.Structure):
    """bfp8_gemm_problem (include/blockfp8_b200.h)."""
    _fields_ = [
        ("a", ctypes.c_void_p), ("lda", ctypes.c_int64),
        ("b", ctypes.c_void_p), ("ldb", ctypes.c_int64),
        ("sa", ctypes.c_void_p), ("sa_m", ctypes.c_int64), ("sa_k", ctypes.c_int64),
        ("sb", ctypes.c_void_p), ("sb_n", ctypes.c_int64), ("sb_k", ctypes.c_int64),
        ("c", ctypes.c_void_p), ("ldc", ctypes.c_int64),
        ("M", ctypes.c_int), ("N", ctypes.c_int), ("K", ctypes.c_int),
        ("eps", ctypes.c_float),
    ]


class Plan(ctypes.Structure):
    """bfp8_plan."""
    _fields_ = [("config", ctypes.c_int), ("splits", ctypes.c_int), ("fused", ctypes.c_int)]

    def __repr__(self):
        return f"Plan(config={self.config}, splits={self.splits}, fused={self.fused})"


class QuantProblem(ctypes.Structure):
    """bfp8_quant_problem."""
    _fields_ = [
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
        ("q", ctypes.c_void_p), ("ldq", ctypes.c_int64),
        ("s", ctypes.c_void_p), ("s_m", ctypes.c_int64), ("s_k", ctypes.c_int64),
        ("M", ctypes.c_int), ("K", ctypes.c_int), ("eps", ctypes.c_float),
    ]


class RmsNormQuantProblem(ctypes.Structure):
    """bfp8_rmsnorm_quant_problem."""
    _fields_ = [
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
        ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64),
        ("residual_out", ctypes.c_void_p), ("ldro", ctypes.c_int64),
        ("weight", ctypes.c_void_p),
        ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
        ("q", ctypes.c_void_p), ("ldq", ctypes.c_int64),
        ("s", ctypes.c_void_p), ("s_m", ctypes.c_int64), ("s_k", ctypes.c_int64),
        ("M", ctypes.c_int), ("H", ctypes.c_int),
        ("variance_epsilon", ctypes.c_float), ("eps", ctypes.c_float),
    ]


class SiluMulQuantProblem(ctypes.Structure):
    """bfp8_silu_mul_quant_problem."""
    _fields_ = [
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
        ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
        ("q", ctypes.c_void_p), ("ldq", ctypes.c_int64),
        ("s", ctypes.c_void_p), ("s_m", ctypes.c_int64), ("s_k", ctypes.c_int64),
        ("M", ctypes.c_int), ("I", ctypes.c_int), ("eps", ctypes.c_float),
    ]


TP_MAX_RANKS = 8
IPC_HANDLE_BYTES = 64


class TpGroup(ctypes.Structure):
    """bfp8_tp_group: a row-parallel group as one launch sees it."""
    _fields_ = [
        ("world", ctypes.c_int), ("rank", ctypes.c_int), ("wait", ctypes.c_int),
        ("partials", ctypes.c_void_p * TP_MAX_RANKS),
        ("counters", ctypes.c_void_p * TP_MAX_RANKS),
        ("out", ctypes.c_void_p * TP_MAX_RANKS),
    ]


# Every function the header declares, with its ctypes signature.
_SIGNATURES = {
    "bfp8_abi_version": ([], ctypes.c_int),
    "bfp8_last_error": ([], ctypes.c_char_p),
    "bfp8_num_configs": ([], ctypes.c_int),
    "bfp8_config_name": ([ctypes.c_int], ctypes.c_char_p),
    "bfp8_num_fused_configs": ([], ctypes.c_int),
    "bfp8_fused_config_name": ([ctypes.c_int], ctypes.c_char_p),
    "bfp8_choose_plan": ([ctypes.c_int] * 4, Plan),
    "bfp8_choose_fused_plan": ([ctypes.c_int] * 4, Plan),
    "bfp8_prefers_fused": ([ctypes.c_int] * 3, ctypes.c_int),
    "bfp8_choose_tp_plan": ([ctypes.c_int] * 5, Plan),
    "bfp8_set_weight_prefetch": ([ctypes.c_int], ctypes.c_int),
    "bfp8_plan_shape": ([ctypes.POINTER(GemmProblem), Plan, ctypes.POINTER(ctypes.c_int),
                         ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "bfp8_workspace_bytes": ([ctypes.POINTER(GemmProblem), Plan], ctypes.c_int64),
    "bfp8_counters_needed": ([ctypes.POINTER(GemmProblem), Plan], ctypes.c_int),
    "bfp8_launch_gemm": ([ctypes.POINTER(GemmProblem), Plan, ctypes.c_void_p, ctypes.c_void_p,
                          ctypes.c_void_p], ctypes.c_int),
    "bfp8_launch_gemm_noalloc": ([ctypes.POINTER(GemmProblem), Plan, ctypes.c_void_p], ctypes.c_int),
    "bfp8_tp_tiles": ([ctypes.POINTER(GemmProblem), Plan], ctypes.c_int),
    "bfp8_tp_partial_bytes": ([ctypes.POINTER(GemmProblem), Plan, ctypes.c_int], ctypes.c_int64),
    "bfp8_launch_gemm_tp": ([ctypes.POINTER(GemmProblem), Plan, ctypes.c_void_p, ctypes.c_void_p,
                             ctypes.POINTER(TpGroup), ctypes.c_void_p], ctypes.c_int),
    "bfp8_tp_alloc": ([ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p], ctypes.c_int),
    "bfp8_tp_open": ([ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "bfp8_tp_close": ([ctypes.c_void_p], ctypes.c_int),
    "bfp8_tp_free": ([ctypes.c_void_p], ctypes.c_int),
    "bfp8_launch_quantize": ([ctypes.POINTER(QuantProblem), ctypes.c_void_p], ctypes.c_int),
    "bfp8_launch_rmsnorm_quant": ([ctypes.POINTER(RmsNormQuantProblem), ctypes.c_void_p], ctypes.c_int),
    "bfp8_launch_silu_mul_quant": ([ctypes.POINTER(SiluMulQuantProblem), ctypes.c_void_p], ctypes.c_int),
    "bfp8_device_status": ([ctypes.c_int], ctypes.c_int64),
    "bfp8_probe_mma": ([ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                        ctypes.POINTER(ctypes.c_double)], ctypes.c_int),
    "bfp8_probe_hbm_read": ([ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.POINTER(ctypes.c_double)],
                            ctypes.c_int),
    "bfp8_probe_block": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
    "bfp8_probe_quantizer": ([ctypes.c_float, ctypes.POINTER(ctypes.c_ulonglong), ctypes.POINTER(ctypes.c_ulonglong)],
                             ctypes.c_int),
    "bfp8_probe_scale": ([ctypes.POINTER(ctypes.c_ulonglong), ctypes.POINTER(ctypes.c_ulonglong)], ctypes.c_int),
}

_capi = None
_ops_loaded = False


def capi() -> ctypes.CDLL:
    """The C ABI library; raises if it has not been built."""
    global _capi
    if _capi is None:
        if not os.path.exists(CAPI_LIB):
            raise RuntimeError(f"native library not built ({CAPI_LIB} missing); "
                               "run python -m blockfp8_b200.build")
        lib = ctypes.CDLL(CAPI_LIB)
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _capi = lib
    return _capi


def capi_loaded() -> bool:
    return _capi is not None


def check(status: int) -> None:
    """Raise RuntimeError with the library's message for a failed call."""
    if status < 0:
        raise RuntimeError(capi().bfp8_last_error().decode())


def load_ops() -> bool:
    """Load _C.so (torch.ops.blockfp8.*) and register the fake kernels once."""
    global _ops_loaded
    if not _ops_loaded and os.path.exists(OPS_LIB):
        capi()  # the same library _C.so links against, loaded first by path
        torch.ops.load_library(OPS_LIB)
        _register_fakes()
        _ops_loaded = True
    return _ops_loaded


def _register_fakes() -> None:
    """Shape functions so torch.compile (and vLLM) can trace through the ops
    (the reference's blockfp8/gemm.py:23-43)."""

    @torch.library.register_fake("blockfp8::gemm")
    def _(a, a_scales, b, b_scales, config=-1, split_k=0):
        return a.new_empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16)

    @torch.library.register_fake("blockfp8::gemm_bf16")
    def _(x, b, b_scales, config=-1, split_k=0, eps=1e-10):
        return x.new_empty((x.shape[0], b.shape[0]), dtype=torch.bfloat16)

    @torch.library.register_fake("blockfp8::linear")
    def _(x, b, b_scales):
        return x.new_empty((x.shape[0], b.shape[0]), dtype=torch.bfloat16)

    @torch.library.register_fake("blockfp8::quantize")
    def _(x, eps=1e-10):
        m, k = x.shape
        q = x.new_empty((m, k), dtype=torch.float8_e4m3fn)
        s = x.new_empty(((k + 127) // 128, m), dtype=torch.float32).t()
        return q, s

    @torch.library.register_fake("blockfp8_b200::rms_norm_quant")
    def _(x, weight, variance_epsilon, residual=None, eps=1e-10):
        m, h = x.shape
        q = x.new_empty((m, h), dtype=torch.float8_e4m3fn)
        s = x.new_empty(((h + 127) // 128, m), dtype=torch.float32).t()
        return q, s, (x.new_empty((m, h)) if residual is not None else x.new_empty((0,)))

    @torch.library.register_fake("blockfp8_b200::silu_mul_quant")
    def _(x, eps=1e-10):
        m, i = x.shape[0], x.shape[1] // 2
        q = x.new_empty((m, i), dtype=torch.float8_e4m3fn)
        s = x.new_empty(((i + 127) // 128, m), dtype=torch.float32).t()
        return q, s


def device_status(reset: bool = False) -> int:
    """Watchdog word of the current device (0 = no kernel gave up a wait)."""
    v = capi().bfp8_device_status(1 if reset else 0)
    check(v if v < 0 else 0)
    return v


def probe_mma(n: int = 256, iters: int = 2000) -> tuple[float, float]:
    """(TFLOP/s, multiply-adds per clock per SM) of back-to-back 128 x n x 32
    e4m3 tcgen05 MMAs on every SM of the current device."""
    tf, mpc = ctypes.c_double(), ctypes.c_double()
    check(capi().bfp8_probe_mma(n, iters, ctypes.byref(tf), ctypes.byref(mpc)))
    return tf.value, mpc.value


def probe_hbm_read(buf, reps: int = 5) -> float:
    """GB/s of a streaming read of the device tensor `buf` (use more than L2)."""
    gbs = ctypes.c_double()
    check(capi().bfp8_probe_hbm_read(ctypes.c_void_p(buf.data_ptr()), buf.numel() * buf.element_size(), reps,
                                     ctypes.byref(gbs)))
    return gbs.value


def probe_block(a, b):
    """fp32 [128, 32] raw tensor-core partial of e4m3 a [128, 128] @ b [32, 128]^T
    (four K = 32 tcgen05 MMAs), on the current device."""
    import torch
    assert a.shape == (128, 128) and b.shape == (32, 128) and a.is_cuda and b.is_cuda
    d = torch.empty(128, 32, dtype=torch.float32, device=a.device)
    check(capi().bfp8_probe_block(ctypes.c_void_p(a.contiguous().data_ptr()),
                                  ctypes.c_void_p(b.contiguous().data_ptr()), ctypes.c_void_p(d.data_ptr()),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return d


def probe_quantizer(eps: float = 1e-10) -> tuple[int, int]:
    """(mismatching codes, first mismatch) of the quantizer's fast path against
    the reference's division sequence over the whole bf16 input domain."""
    bad, first = ctypes.c_ulonglong(), ctypes.c_ulonglong()
    check(capi().bfp8_probe_quantizer(eps, ctypes.byref(bad), ctypes.byref(first)))
    return bad.value, first.value


def probe_scale() -> tuple[int, int]:
    """(mismatching scales, first mismatch + 1) of the quantizer's amax / 448
    against the IEEE division over every finite non-negative float."""
    bad, first = ctypes.c_ulonglong(), ctypes.c_ulonglong()
    check(capi().bfp8_probe_scale(ctypes.byref(bad), ctypes.byref(first)))
    return bad.value, first.value
