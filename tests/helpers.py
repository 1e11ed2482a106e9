"""Shared test helpers: seeded operands and comparisons against the CPU oracle."""

import re

import numpy as np
import torch

from oracle import oracle as O

FP8 = torch.float8_e4m3fn
# Parity contract for the GEMM output: |C - ref| <= RTOL |ref| + ATOL max|ref|.
RTOL = 1e-2
ATOL_REL_MAX = 1e-2


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def codes(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().float().numpy()


def integer_operands(m, n, k, seed=0, dev="cuda"):
    """|a|, |b| <= 4 integers, scales in 2^[-1, 1]: every partial sum is exact
    in the MMA and in fp32 (the reference's tests/test_gemm_gpu.py:40-48)."""
    g = gen(seed)
    kb, nb = -(-k // 128), -(-n // 128)
    a = torch.randint(-4, 5, (m, k), generator=g).float().to(FP8)
    b = torch.randint(-4, 5, (n, k), generator=g).float().to(FP8)
    sa = torch.exp2(torch.randint(-1, 2, (m, kb), generator=g).float())
    sb = torch.exp2(torch.randint(-1, 2, (nb, kb), generator=g).float())
    return a.to(dev), sa.to(dev), b.to(dev), sb.to(dev)


def realistic_operands(m, n, k, seed=0, col_major=True, dev="cuda"):
    """x ~ N(0, 1), w ~ N(0, 0.02) on a CPU generator, quantized by the oracle."""
    g = gen(seed)
    x = torch.randn(m, k, generator=g)
    w = torch.randn(n, k, generator=g) * 0.02
    a, sa = O.quantize_activations(x.numpy(), column_major_scales=col_major)
    b, sb = O.quantize_weights(w.numpy())
    a_t = torch.from_numpy(a).view(FP8).to(dev)
    sa_t = torch.from_numpy(np.ascontiguousarray(sa.T)).t().to(dev) if col_major else \
        torch.from_numpy(sa).to(dev)
    return a_t, sa_t, torch.from_numpy(b).view(FP8).to(dev), torch.from_numpy(sb).to(dev)


def bf16_activations(m, k, seed=0, ties=False, scale=2.0):
    """Seeded bf16 activations (CPU).  ties=True gives every 128-wide group an
    amax of 448 * 2^j, so x / scale is exact and many values fall exactly
    halfway between two e4m3 values (the reference's
    tests/test_gemm_gpu.py:279-292 construction)."""
    g = gen(seed)
    x = torch.randn(m, k, generator=g) * scale
    if ties:
        kb = -(-k // 128)
        xp = torch.nn.functional.pad(x, (0, kb * 128 - k)).view(m, kb, 128)
        top = 448.0 * torch.exp2(torch.randint(-12, 12, (m, kb, 1), generator=g).float())
        xp = xp / xp.abs().amax(dim=2, keepdim=True).clamp_min(1e-30) * top
        xp[:, :, :1] = top * torch.sign(torch.randn(m, kb, 1, generator=g))
        x = xp.reshape(m, kb * 128)[:, :k]
    return x.to(torch.bfloat16).contiguous()


def oracle_gemm(a, sa, b, sb, absolute=False) -> np.ndarray:
    return O.reference_gemm(codes(a), f32(sa), codes(b), f32(sb), absolute=absolute)


def oracle_quant(x: torch.Tensor, eps=1e-10):
    """(codes, scales) of the oracle for bf16 x."""
    return O.quantize_activations(bf16_bits(x), eps=eps)


def assert_exact(c: torch.Tensor, ref: np.ndarray) -> None:
    got = bf16_bits(c)
    want = O.f64_to_bf16_bits(ref)
    bad = np.nonzero(got != want)
    assert bad[0].size == 0, f"{bad[0].size} of {got.size} outputs differ, first at {bad[0][0], bad[1][0]}"


def assert_close(c: torch.Tensor, ref: np.ndarray, rtol=RTOL, atol_rel_max=ATOL_REL_MAX) -> float:
    """The parity tolerance; returns the worst error as a fraction of it."""
    got = c.detach().cpu().double().numpy()
    tol = rtol * np.abs(ref) + atol_rel_max * max(np.abs(ref).max(), 1e-300)
    err = np.abs(got - ref)
    worst = float((err / tol).max()) if ref.size else 0.0
    assert np.all(np.isfinite(got)), "non-finite output"
    assert worst <= 1.0, f"error exceeds the tolerance by {worst:.3g}x"
    return worst


def token_limit(name: str):
    """Most tokens (M) a weight-streaming configuration ("w128d<BN>")
    handles; None for the tile configurations, which take any M."""
    m = re.fullmatch(r"w128d(\d+)", name)
    return int(m.group(1)) if m else None


def config_geometry(name: str):
    """(MMA rows of a tile, tile width BN, swapped order) of a configuration
    name: "m<BM>n<BN>..." (activation rows x weight rows), "w128t<BN>..." and
    "w128d<BN>" (weight rows x tokens)."""
    m = re.match(r"([mw])(\d+)[ntd](\d+)", name)
    return int(m.group(2)), int(m.group(3)), m.group(1) == "w"
