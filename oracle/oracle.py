"""CPU parity oracle for blockfp8's hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only to check or time against it.  The blockfp8_b200
package never imports it, so a missing or broken oracle can never stand in
for the CUDA path.

Restated from the reference (simon-jd/blockfp8), in numpy + a small C
library (bfp8_oracle.c) for the bit-level float8 rounding:

  quantize_activations   blockfp8/quant.py:39-64 (1 x 128 groups, scale =
                         max(amax, eps) / 448 by true division, M-major scales
                         by default)
  quantize_weights       blockfp8/quant.py:67-79 (128 x 128 blocks)
  reference_gemm         blockfp8/reference.py:20-46 (float64, block by block
                         along K; each 128-wide block sum is exact in float64,
                         so BLAS may sum it in any order)
  dequantize_*           blockfp8/reference.py:49-59
  error_bound, acc_gamma blockfp8/reference.py:62-82 (the reference's
                         worst-case model of its sm_89 MMA, 13 kept bits)

Arrays are numpy: float8 codes travel as uint8, bf16 values as uint16 bits.
The oracle is pinned against vectors produced by the reference itself
(tests/golden/, made by tests/golden/make_golden.py) and against the
reference's own known-answer tests (tests/test_oracle.py).
"""

import ctypes
import os

import numpy as np

from . import build as _build

FP8_MAX = 448.0
GROUP_K = 128
BLOCK_N = 128

_lib = None


def cdiv(a: int, b: int) -> int:
    return -(-a // b)


def lib() -> ctypes.CDLL:
    """The compiled C half of the oracle (built on first use if missing)."""
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        f32p = ctypes.POINTER(ctypes.c_float)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        i64 = ctypes.c_int64
        L.oracle_quantize_activations.argtypes = [f32p, i64, i64, i64, ctypes.c_float, u8p, i64,
                                                  f32p, i64, i64]
        L.oracle_quantize_activations.restype = None
        L.oracle_quantize_weights.argtypes = [f32p, i64, i64, i64, ctypes.c_float, u8p, i64, f32p]
        L.oracle_quantize_weights.restype = None
        L.oracle_e4m3_decode.argtypes = [u8p, i64, f32p]
        L.oracle_e4m3_decode.restype = None
        L.oracle_e4m3_decode_f64.argtypes = [u8p, i64, ctypes.POINTER(ctypes.c_double)]
        L.oracle_e4m3_decode_f64.restype = None
        L.oracle_e4m3_from_float.argtypes = [ctypes.c_float]
        L.oracle_e4m3_from_float.restype = ctypes.c_uint8
        _lib = L
    return _lib


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


# ---- bf16 / e4m3 helpers ---------------------------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32, exactly."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    """float8_e4m3fn codes (uint8) -> float32, exactly."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    out = np.empty(c.shape, dtype=np.float32)
    lib().oracle_e4m3_decode(_ptr(c, ctypes.c_uint8), c.size, _ptr(out, ctypes.c_float))
    return out


def e4m3_decode_f64(codes: np.ndarray) -> np.ndarray:
    """float8_e4m3fn codes (uint8) -> float64, exactly."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    out = np.empty(c.shape, dtype=np.float64)
    lib().oracle_e4m3_decode_f64(_ptr(c, ctypes.c_uint8), c.size, _ptr(out, ctypes.c_double))
    return out


def e4m3_encode(values: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn codes, round to nearest even (saturating)."""
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    f = lib().oracle_e4m3_from_float
    return np.array([f(float(x)) for x in v], dtype=np.uint8).reshape(np.shape(values))


# ---- quantizers --------------------------------------------------------------

def quantize_activations(x: np.ndarray, eps: float = 1e-10, column_major_scales: bool = True):
    """x [M, K] (float32, or bf16 bits as uint16) -> (codes uint8 [M, K],
    scales float32 [M, ceil(K/128)]).  quant.py:39-64.  With
    column_major_scales the scale array is M-contiguous (Fortran order), the
    reference's default layout."""
    if x.ndim != 2:
        raise ValueError(f"x must be 2-D [M, K], got shape {x.shape}")
    xf = bf16_bits_to_f32(x) if x.dtype == np.uint16 else np.asarray(x, dtype=np.float32)
    xf = np.ascontiguousarray(xf)
    m, k = xf.shape
    kb = cdiv(k, GROUP_K)
    q = np.empty((m, k), dtype=np.uint8)
    if column_major_scales:
        s = np.empty((m, kb), dtype=np.float32, order="F")
        s_m, s_k = 1, m
    else:
        s = np.empty((m, kb), dtype=np.float32)
        s_m, s_k = kb, 1
    lib().oracle_quantize_activations(_ptr(xf, ctypes.c_float), m, k, k, eps,
                                      _ptr(q, ctypes.c_uint8), k, _ptr(s, ctypes.c_float), s_m, s_k)
    return q, s


def quantize_weights(w: np.ndarray, eps: float = 1e-10):
    """w [N, K] float32 -> (codes uint8 [N, K], scales float32 [nb, kb]).
    quant.py:67-79."""
    if w.ndim != 2:
        raise ValueError(f"w must be 2-D [N, K], got shape {w.shape}")
    wf = np.ascontiguousarray(w, dtype=np.float32)
    n, k = wf.shape
    q = np.empty((n, k), dtype=np.uint8)
    s = np.empty((cdiv(n, BLOCK_N), cdiv(k, GROUP_K)), dtype=np.float32)
    lib().oracle_quantize_weights(_ptr(wf, ctypes.c_float), n, k, k, eps,
                                  _ptr(q, ctypes.c_uint8), k, _ptr(s, ctypes.c_float))
    return q, s


# ---- the float64 reference GEMM ---------------------------------------------

def _expand_b_scales(b_scales: np.ndarray, n: int) -> np.ndarray:
    return np.repeat(b_scales, BLOCK_N, axis=0)[:n]


def reference_gemm(a_q, a_scales, b_q, b_scales, absolute: bool = False) -> np.ndarray:
    """C [M, N] float64 = sum_kb sa[m,kb] sb[n//128,kb] sum_{k in kb} a[m,k] b[n,k].
    reference.py:20-46, including its operation order per block:
    c += block * (sa * sb), each step rounded separately in float64."""
    m, k = a_q.shape
    n = b_q.shape[0]
    a = e4m3_decode_f64(a_q)
    b = e4m3_decode_f64(b_q)
    sa = np.asarray(a_scales, dtype=np.float64)
    sb = _expand_b_scales(np.asarray(b_scales, dtype=np.float64), n)
    if absolute:
        a, b, sa, sb = np.abs(a), np.abs(b), np.abs(sa), np.abs(sb)
    c = np.zeros((m, n), dtype=np.float64)
    for j in range(cdiv(k, GROUP_K)):
        k0, k1 = j * GROUP_K, min(k, (j + 1) * GROUP_K)
        block = a[:, k0:k1] @ b[:, k0:k1].T  # exact: multiples of 2^-18 below 2^25
        c += block * (sa[:, j:j + 1] * sb[:, j][None, :])
    return c


def dequantize_activations(x_q, scales) -> np.ndarray:
    k = x_q.shape[1]
    s = np.repeat(np.asarray(scales, dtype=np.float64), GROUP_K, axis=1)[:, :k]
    return e4m3_decode(x_q).astype(np.float64) * s


def dequantize_weights(w_q, scales) -> np.ndarray:
    n, k = w_q.shape
    s = np.repeat(_expand_b_scales(np.asarray(scales, dtype=np.float64), n), GROUP_K, axis=1)[:, :k]
    return e4m3_decode(w_q).astype(np.float64) * s


# ---- the reference's error model (reference.py:62-82) ------------------------

MMA_FRACTION_BITS = 13
BF16_U = 2.0 ** -8
FP32_U = 2.0 ** -24


def acc_gamma(k: int, fraction_bits: int = MMA_FRACTION_BITS) -> float:
    kb = cdiv(k, 128)
    return 4 * 33 * 2.0 ** -fraction_bits + (4 + 3 * kb) * FP32_U


def error_bound(c_exact, c_abs, k: int, fraction_bits: int = MMA_FRACTION_BITS):
    acc = acc_gamma(k, fraction_bits) * c_abs
    return BF16_U * (np.abs(c_exact) + acc) + acc + np.finfo(np.float32).tiny


# ---- float64 -> bf16 as torch rounds it (via float32, each step RNE) ---------

def f64_to_bf16_bits(c: np.ndarray) -> np.ndarray:
    f = np.asarray(c, dtype=np.float64).astype(np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    nan = np.isnan(f)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, np.uint16(0x7FC0), rounded)
