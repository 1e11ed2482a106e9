"""Pin the CPU oracle: against vectors the reference produced (tests/golden/)
and against the reference's own known-answer tests, restated.

The reference tests restated here: blockfp8 tests/test_quant.py:17-94 and
tests/test_reference.py:14-58.
"""

import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def quant():
    return np.load(os.path.join(GOLDEN, "quant.npz"))


@pytest.fixture(scope="module")
def gemm():
    return np.load(os.path.join(GOLDEN, "gemm.npz"))


# ---- golden vectors ----------------------------------------------------------

def test_activation_quantizer_matches_reference_vectors_bitwise(quant):
    for i in range(int(quant["act_count"])):
        x = quant[f"act{i}_x_bf16"]
        for j, eps in enumerate(quant["act_eps"]):
            q, s = O.quantize_activations(x, eps=float(eps))
            assert np.array_equal(q, quant[f"act{i}_eps{j}_q"]), (i, j)
            assert np.array_equal(s.view(np.uint32), quant[f"act{i}_eps{j}_s"].view(np.uint32)), (i, j)
            assert s.strides == (4, 4 * x.shape[0])  # M-major, like the reference's default


def test_float32_activations_zero_group_outliers_and_tail(quant):
    q, s = O.quantize_activations(quant["actf_x"])
    assert np.array_equal(q, quant["actf_q"])
    assert np.array_equal(s, quant["actf_s"])
    _, s_row = O.quantize_activations(quant["actf_x"], column_major_scales=False)
    assert s_row.flags.c_contiguous and np.array_equal(s_row, quant["actf_s_rowmajor"])


def test_true_division_known_answer(quant):
    q, s = O.quantize_activations(quant["kat_div_x"])
    assert np.array_equal(s, quant["kat_div_s"]) and np.array_equal(q, quant["kat_div_q"])
    amax = np.float32(5.03125)
    assert s[0, 0] == amax / np.float32(448.0)
    assert s[0, 0] != amax * np.float32(1.0 / 448.0)  # the multiply would be one ulp off


def test_weight_quantizer_matches_reference_vectors(quant):
    for i in range(int(quant["wgt_count"])):
        q, s = O.quantize_weights(quant[f"wgt{i}_w"])
        assert np.array_equal(q, quant[f"wgt{i}_q"]) and np.array_equal(s, quant[f"wgt{i}_s"]), i


def test_reference_gemm_matches_reference_vectors(gemm):
    for i in range(int(gemm["g_count"])):
        a, sa, b, sb = gemm[f"g{i}_a"], gemm[f"g{i}_sa"], gemm[f"g{i}_b"], gemm[f"g{i}_sb"]
        c = O.reference_gemm(a, sa, b, sb)
        assert np.array_equal(c, gemm[f"g{i}_c"]), i
        assert np.array_equal(O.reference_gemm(a, sa, b, sb, absolute=True), gemm[f"g{i}_cabs"]), i
        assert np.array_equal(O.f64_to_bf16_bits(c), gemm[f"g{i}_c_bf16"]), i


def test_error_model_numbers(gemm):
    assert np.allclose([O.acc_gamma(k) for k in (128, 4096, 12288)], gemm["acc_gamma"], rtol=0, atol=0)


# ---- the reference's known-answer tests, restated on the oracle ---------------

def _rand(m, k, seed):
    return (np.random.default_rng(seed).standard_normal((m, k)) * 3).astype(np.float32)


def test_scales_are_group_amax_over_fp8_max():
    x = _rand(5, 384, 0)
    _, s = O.quantize_activations(x)
    expect = np.stack([np.abs(x[:, i * 128:(i + 1) * 128]).max(axis=1) for i in range(3)], axis=1)
    assert np.array_equal(s, expect / np.float32(448.0))


def test_group_max_maps_to_fp8_max():
    q, _ = O.quantize_activations(_rand(7, 256, 1))
    qa = np.abs(O.e4m3_decode(q)).reshape(7, 2, 128).max(axis=2)
    assert np.all(qa == 448.0)


def test_round_trip_error_within_half_ulp():
    x = _rand(9, 512, 2)
    q, s = O.quantize_activations(x)
    err = np.abs(O.dequantize_activations(q, s) - x.astype(np.float64))
    s_full = np.repeat(s.astype(np.float64), 128, axis=1)
    bound = np.maximum(np.abs(x.astype(np.float64)) * 2.0 ** -4, s_full * 2.0 ** -10)
    assert np.all(err <= bound * (1 + 1e-6))


def test_zero_group_gets_eps_scale_and_zero_codes():
    x = _rand(3, 256, 3)
    x[1, 128:] = 0
    q, s = O.quantize_activations(x, eps=1e-10)
    assert s[1, 1] == np.float32(1e-10) / np.float32(448.0)
    assert np.all(q[1, 128:] == 0)


def test_exact_on_integers_with_power_of_two_scales():
    rng = np.random.default_rng(1)
    m, n, k = 4, 136, 272
    ai = rng.integers(-16, 17, (m, k))
    bi = rng.integers(-16, 17, (n, k))
    a_q, b_q = O.e4m3_encode(ai.astype(np.float32)), O.e4m3_encode(bi.astype(np.float32))
    assert np.array_equal(O.e4m3_decode(a_q), ai.astype(np.float32))
    ea, eb = rng.integers(-6, 7, (m, 3)), rng.integers(-6, 7, (2, 3))
    c = O.reference_gemm(a_q, np.exp2(ea).astype(np.float32), b_q, np.exp2(eb).astype(np.float32))
    exact = np.zeros((m, n))
    for kb in range(3):
        sl = slice(kb * 128, min(k, kb * 128 + 128))
        e = ea[:, kb][:, None] + eb[np.arange(n) // 128, kb][None, :]
        exact += (ai[:, sl] @ bi[:, sl].T).astype(np.float64) * np.exp2(e.astype(np.float64))
    assert np.array_equal(c, exact)


def test_extreme_values_exact_per_block():
    a_q = np.zeros((1, 128), np.uint8)
    b_q = np.zeros((8, 128), np.uint8)
    a_q[0, 0] = b_q[0, 0] = O.e4m3_encode(np.float32([448.0]))[0]
    a_q[0, 1] = b_q[0, 1] = O.e4m3_encode(np.float32([2.0 ** -9]))[0]
    one = np.ones((1, 1), np.float32)
    assert O.reference_gemm(a_q, one, b_q, one)[0, 0] == 448.0 * 448.0 + 2.0 ** -18


def test_absolute_bounds_the_result():
    rng = np.random.default_rng(2)
    a_q, a_s = O.quantize_activations(rng.standard_normal((3, 256)).astype(np.float32))
    b_q, b_s = O.quantize_weights((rng.standard_normal((128, 256)) * 0.02).astype(np.float32))
    c = O.reference_gemm(a_q, a_s, b_q, b_s)
    assert np.all(np.abs(c) <= O.reference_gemm(a_q, a_s, b_q, b_s, absolute=True))


def test_matches_dequantized_matmul():
    rng = np.random.default_rng(0)
    a_q, a_s = O.quantize_activations(rng.standard_normal((5, 400)).astype(np.float32))
    b_q, b_s = O.quantize_weights((rng.standard_normal((264, 400)) * 0.02).astype(np.float32))
    c = O.reference_gemm(a_q, a_s, b_q, b_s)
    expect = O.dequantize_activations(a_q, a_s) @ O.dequantize_weights(b_q, b_s).T
    assert np.allclose(c, expect, rtol=1e-12, atol=1e-12)


def test_rejects_bad_input():
    with pytest.raises(ValueError):
        O.quantize_activations(np.zeros(128, np.float32))
    with pytest.raises(ValueError):
        O.quantize_weights(np.zeros(128, np.float32))
