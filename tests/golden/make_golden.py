"""Generate the golden vectors in tests/golden/ from the reference itself.

Run in a container that has the reference checkout (simon-jd/blockfp8):

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's pure-PyTorch oracle (blockfp8/quant.py,
blockfp8/reference.py) under the private module name `_ref_blockfp8`, so it
cannot collide with this repository's own `blockfp8` package, and records
inputs and outputs as compressed .npz files.  Inputs are stored too, so the
fixtures do not depend on torch's random number streams staying the same.

Contents (every array is plain numpy; float8 as uint8 codes, bf16 as uint16):
  quant_act.npz     quantize_activations on bf16 and float32 inputs: the
                    reference GPU test shapes (blockfp8 tests/test_gemm_gpu.py
                    :339) scaled down, with and without exact e4m3 ties
                    (:279-292), eps in {1e-10, 1e-2}, a zero group, a K tail,
                    and the true-division known answer amax = 5.03125
                    (tests/test_quant.py:61-68)
  quant_wgt.npz     quantize_weights with ragged blocks (tests/test_quant.py:80-87)
  gemm.npz          reference_gemm (float64) and its absolute variant on
                    realistic, integer/power-of-two, tail and extreme operands
                    (tests/test_reference.py:7-51)
"""

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def import_reference(root: str):
    pkg_dir = os.path.join(root, "blockfp8")
    spec = importlib.util.spec_from_file_location(
        "_ref_blockfp8", os.path.join(pkg_dir, "__init__.py"),
        submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["_ref_blockfp8"] = mod
    spec.loader.exec_module(mod)  # gemm.py loads _C.so lazily; nothing native is needed
    return mod


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def codes(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy().copy()


def bf16_activations(m, k, seed, ties):
    """Seeded bf16 activations; ties=True gives every 128-wide group an amax
    of 448 * 2^j so x / scale is exact and many values fall exactly halfway
    between two e4m3 values (the construction of the reference's
    tests/test_gemm_gpu.py:279-292, on a CPU generator)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g) * 2
    if ties:
        kb = -(-k // 128)
        xp = torch.nn.functional.pad(x, (0, kb * 128 - k)).view(m, kb, 128)
        top = 448.0 * torch.exp2(torch.randint(-12, 12, (m, kb, 1), generator=g).float())
        xp = xp / xp.abs().amax(dim=2, keepdim=True) * top
        xp[:, :, :1] = top * torch.sign(torch.randn(m, kb, 1, generator=g))
        x = xp.reshape(m, kb * 128)[:, :k]
    x = x.to(torch.bfloat16).contiguous()
    x[0, :16] = 0.0
    return x


def main(root: str) -> None:
    ref = import_reference(root)
    out = {}

    # ---- activations, bf16 input
    cases = []
    for shape in [(1, 128), (7, 272), (33, 640), (64, 1040)]:
        for ties in (False, True):
            cases.append((shape, ties, 15 + len(cases)))
    for i, ((m, k), ties, seed) in enumerate(cases):
        x = bf16_activations(m, k, seed, ties)
        out[f"act{i}_x_bf16"] = bf16_bits(x)
        for j, eps in enumerate((1e-10, 1e-2)):
            q, s = ref.quantize_activations(x, eps=eps)
            assert s.stride() == (1, m)
            out[f"act{i}_eps{j}_q"] = codes(q)
            out[f"act{i}_eps{j}_s"] = s.contiguous().numpy()
    out["act_eps"] = np.array([1e-10, 1e-2])
    out["act_count"] = np.array(len(cases))

    # ---- activations, float32 input, incl. zero group, outliers, K tail
    g = torch.Generator().manual_seed(3)
    xf = torch.randn(5, 200, generator=g) * 3
    xf[1, 128:] = 0.0
    xf[2, 7] = 1e4
    xf[3, :] = 1e-38
    out["actf_x"] = xf.numpy().copy()
    q, s = ref.quantize_activations(xf)
    out["actf_q"], out["actf_s"] = codes(q), s.contiguous().numpy()
    q, s = ref.quantize_activations(xf, column_major_scales=False)
    assert s.stride() == (2, 1)
    out["actf_s_rowmajor"] = s.numpy().copy()

    # the true-division known answer
    x = torch.zeros(1, 128)
    x[0, 0] = 5.03125
    q, s = ref.quantize_activations(x)
    out["kat_div_x"], out["kat_div_q"], out["kat_div_s"] = x.numpy().copy(), codes(q), s.numpy().copy()

    # ---- weights
    for i, (n, k) in enumerate([(200, 272), (136, 400), (256, 128)]):
        g = torch.Generator().manual_seed(6 + i)
        w = torch.randn(n, k, generator=g) * 0.02
        q, s = ref.quantize_weights(w)
        out[f"wgt{i}_w"], out[f"wgt{i}_q"], out[f"wgt{i}_s"] = w.numpy().copy(), codes(q), s.numpy().copy()
    out["wgt_count"] = np.array(3)
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **out)

    # ---- GEMM
    gm = {}
    gcases = []
    for (m, n, k, seed) in [(5, 264, 400, 0), (33, 264, 272, 1), (17, 256, 512, 2), (1, 128, 128, 3)]:
        g = torch.Generator().manual_seed(seed)
        a_q, a_s = ref.quantize_activations(torch.randn(m, k, generator=g))
        b_q, b_s = ref.quantize_weights(torch.randn(n, k, generator=g) * 0.02)
        gcases.append((a_q, a_s, b_q, b_s))
    # integer operands with power-of-two scales (tests/test_reference.py:21-39)
    g = torch.Generator().manual_seed(1)
    m, n, k = 4, 136, 272
    ai = torch.randint(-16, 17, (m, k), generator=g)
    bi = torch.randint(-16, 17, (n, k), generator=g)
    ea = torch.randint(-6, 7, (m, 3), generator=g)
    eb = torch.randint(-6, 7, (2, 3), generator=g)
    gcases.append((ai.float().to(torch.float8_e4m3fn), torch.exp2(ea.float()),
                   bi.float().to(torch.float8_e4m3fn), torch.exp2(eb.float())))
    # extreme values (tests/test_reference.py:42-51 and tests/test_gemm_gpu.py:205-214)
    g = torch.Generator().manual_seed(8)
    choices = torch.tensor([448.0, -448.0, 2.0 ** -9, -(2.0 ** -9), 2.0 ** -6, 0.0])
    a = choices[torch.randint(0, 6, (32, 512), generator=g)].to(torch.float8_e4m3fn)
    b = choices[torch.randint(0, 6, (128, 512), generator=g)].to(torch.float8_e4m3fn)
    gcases.append((a, torch.full((32, 4), 2.0 ** -10), b, torch.full((1, 4), 2.0 ** -8)))
    for i, (a_q, a_s, b_q, b_s) in enumerate(gcases):
        gm[f"g{i}_a"], gm[f"g{i}_sa"] = codes(a_q), a_s.contiguous().numpy()
        gm[f"g{i}_b"], gm[f"g{i}_sb"] = codes(b_q), b_s.contiguous().numpy()
        gm[f"g{i}_c"] = ref.reference_gemm(a_q, a_s, b_q, b_s).numpy()
        gm[f"g{i}_cabs"] = ref.reference_gemm(a_q, a_s, b_q, b_s, absolute=True).numpy()
        gm[f"g{i}_c_bf16"] = bf16_bits(gm_t := ref.reference_gemm(a_q, a_s, b_q, b_s).to(torch.bfloat16))
        del gm_t
    gm["g_count"] = np.array(len(gcases))
    # the error model's numbers for two K values
    gm["acc_gamma"] = np.array([ref.reference.acc_gamma(k) for k in (128, 4096, 12288)])
    np.savez_compressed(os.path.join(HERE, "gemm.npz"), **gm)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("BLOCKFP8_REFERENCE", ""))
