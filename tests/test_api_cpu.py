"""CPU tests of the drop-in boundary: argument validation (the reference's
tests/test_validation.py restated), the C ABI library (loads, exports every
symbol include/blockfp8_b200.h declares, planner and sizing answers), the
torch op schemas, and the public torch helpers against the golden vectors."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

import blockfp8
import blockfp8_b200
from helpers import config_geometry, token_limit
from blockfp8_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
FP8 = torch.float8_e4m3fn


# ---- validation ----------------------------------------------------------------

def _args(m=4, n=256, k=512, col_major=True):
    a_q = torch.zeros(m, k).to(FP8)
    b_q = torch.zeros(n, k).to(FP8)
    kb, nb = -(-k // 128), -(-n // 128)
    a_s = torch.ones(kb, m).t() if col_major else torch.ones(m, kb)
    return a_q, a_s, b_q, torch.ones(nb, kb)


@pytest.mark.parametrize("col_major", [True, False])
def test_valid_args(col_major):
    assert blockfp8.check_gemm_args(*_args(col_major=col_major), torch.bfloat16) == (4, 256, 512)


def test_tails_are_accepted():
    assert blockfp8.check_gemm_args(*_args(m=3, n=136, k=144), torch.bfloat16) == (3, 136, 144)


@pytest.mark.parametrize("mutate, match", [
    (lambda a: (a[0].float(), *a[1:]), "float8_e4m3fn"),
    (lambda a: (a[0][:, :500], a[1], a[2], a[3]), "K mismatch"),
    (lambda a: (a[0], a[1], a[2].to(torch.float8_e5m2), a[3]), "float8_e4m3fn"),
    (lambda a: (a[0], a[1].double(), a[2], a[3]), "a_scales"),
    (lambda a: (a[0], a[1][:, :3], a[2], a[3]), "a_scales"),
    (lambda a: (a[0], a[1], a[2], a[3][:1]), "b_scales"),
    (lambda a: (a[0].t().contiguous().t(), *a[1:]), "row-major"),
])
def test_rejects(mutate, match):
    with pytest.raises(ValueError, match=match):
        blockfp8.check_gemm_args(*mutate(_args()), torch.bfloat16)


def test_rejects_unaligned_k_and_n():
    with pytest.raises(ValueError, match="K must be"):
        blockfp8.check_gemm_args(*_args(k=200), torch.bfloat16)
    with pytest.raises(ValueError, match="N must be"):
        blockfp8.check_gemm_args(*_args(n=100), torch.bfloat16)


def test_rejects_other_output_dtypes():
    with pytest.raises(ValueError, match="out_dtype"):
        blockfp8.check_gemm_args(*_args(), torch.float16)


def test_cpu_tensors_point_to_the_reference():
    with pytest.raises(ValueError, match="reference_gemm"):
        blockfp8.gemm(*_args())


def test_bf16_entry_points_reject_cpu_and_bad_layouts():
    b_q, b_s = _args()[2:]
    with pytest.raises(ValueError):
        blockfp8.linear(torch.zeros(2, 512, dtype=torch.bfloat16), b_q, b_s)  # CPU tensor
    with pytest.raises(ValueError):
        blockfp8.gemm_bf16(torch.zeros(2, 512), b_q, b_s)  # float32
    with pytest.raises(ValueError, match="CUDA"):
        blockfp8.gemm_bf16(torch.zeros(2, 512, dtype=torch.bfloat16), b_q, b_s)


# ---- the API surface -------------------------------------------------------------

def test_public_names_match_the_reference_api():
    expected = {"BLOCK_N", "FP8_DTYPE", "FP8_MAX", "GROUP_K", "check_gemm_args", "configs",
                "dequantize_activations", "dequantize_weights", "error_bound", "fused_configs",
                "gemm", "gemm_bf16", "linear", "native_available", "prefers_fused",
                "quantize_activations", "quantize_cuda", "quantize_weights", "reference_gemm"}
    assert expected <= set(blockfp8.__all__)
    for name in expected:
        assert getattr(blockfp8, name) is getattr(blockfp8_b200, name)
    from blockfp8.reference import BF16_U  # submodule aliases exist
    assert BF16_U == 2.0 ** -8


def test_torch_helpers_match_the_reference_vectors():
    """quantize_activations / quantize_weights / reference_gemm of the public
    API give the reference's bits (they prepare operands; not the hot path)."""
    g = np.load(os.path.join(GOLDEN, "quant.npz"))
    for i in range(int(g["act_count"])):
        x = torch.from_numpy(g[f"act{i}_x_bf16"].view(np.int16)).view(torch.bfloat16)
        for j, eps in enumerate(g["act_eps"]):
            q, s = blockfp8.quantize_activations(x, eps=float(eps))
            assert np.array_equal(q.view(torch.uint8).numpy(), g[f"act{i}_eps{j}_q"])
            assert np.array_equal(s.numpy(), g[f"act{i}_eps{j}_s"]) and s.stride() == (1, x.shape[0])
    for i in range(int(g["wgt_count"])):
        q, s = blockfp8.quantize_weights(torch.from_numpy(g[f"wgt{i}_w"]))
        assert np.array_equal(q.view(torch.uint8).numpy(), g[f"wgt{i}_q"])
        assert np.array_equal(s.numpy(), g[f"wgt{i}_s"])
    gm = np.load(os.path.join(GOLDEN, "gemm.npz"))
    for i in range(int(gm["g_count"])):
        args = [torch.from_numpy(gm[f"g{i}_a"]).view(FP8), torch.from_numpy(gm[f"g{i}_sa"]),
                torch.from_numpy(gm[f"g{i}_b"]).view(FP8), torch.from_numpy(gm[f"g{i}_sb"])]
        assert np.array_equal(blockfp8.reference_gemm(*args).numpy(), gm[f"g{i}_c"])


# ---- the C ABI library ------------------------------------------------------------

def _declared_functions():
    header = open(os.path.join(ROOT, "include", "blockfp8_b200.h")).read()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)
    return sorted(set(re.findall(r"\b(bfp8_[a-z_0-9]+)\s*\(", header)))


def test_c_abi_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_native.CAPI_LIB)
    names = _declared_functions()
    assert len(names) >= 14
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(_native._SIGNATURES), "ctypes signatures out of date with the header"


def test_c_abi_answers_without_a_gpu():
    lib = _native.capi()
    assert lib.bfp8_abi_version() == 1
    n = lib.bfp8_num_configs()
    assert n >= 1 and lib.bfp8_num_fused_configs() >= 1
    names = [lib.bfp8_config_name(i).decode() for i in range(n)]
    assert names == blockfp8.configs()
    assert lib.bfp8_config_name(n) is None
    for m, nn, k in [(1, 6144, 4096), (16, 24576, 4096), (256, 6144, 4096), (8192, 24576, 4096),
                     (3000, 4096, 12288), (33, 264, 272)]:
        plan = lib.bfp8_choose_plan(m, nn, k, 148)
        assert 0 <= plan.config < n and plan.splits != 0 and plan.fused == 0
        assert plan.splits >= 1 or names[plan.config].startswith("w")  # stream-K: the decode configurations
        fplan = lib.bfp8_choose_fused_plan(m, nn, k, 148)
        assert fplan.fused in (1, 2)
        if fplan.fused == 1:  # quantization kernel + the GEMM's own plan: same bits as unfused
            assert (fplan.config, fplan.splits) == (plan.config, plan.splits)
        p = _native.GemmProblem(M=m, N=nn, K=k)
        tiles, kt = ctypes.c_int(), ctypes.c_int()
        assert lib.bfp8_plan_shape(ctypes.byref(p), plan, ctypes.byref(tiles), ctypes.byref(kt)) == 0
        assert kt.value == -(-k // 128)
        ws = lib.bfp8_workspace_bytes(ctypes.byref(p), plan)
        cnt = lib.bfp8_counters_needed(ctypes.byref(p), plan)
        if plan.splits > 0 and token_limit(names[plan.config]) is None:
            splits = -(-kt.value // -(-kt.value // min(plan.splits, kt.value)))
            assert (ws == 0) == (splits == 1) and (cnt == 0) == (splits == 1)
        assert ws >= 0 and cnt >= 0 and (ws == 0) == (cnt == 0)
        # quantization kernel first: q and s live in the front of the workspace
        q_plan = _native.Plan(plan.config, plan.splits, 1)
        assert lib.bfp8_workspace_bytes(ctypes.byref(p), q_plan) >= m * k + ws
        # quantization inside the GEMM: only split-K scratch where the
        # configuration has that variant and a split's K blocks fit its
        # resident operand (64 KB of BN x 128 e4m3 tiles), else as above
        for config in range(n):
            for splits in (1, 2, 4, 8):
                in_plan, q_plan = _native.Plan(config, splits, 2), _native.Plan(config, splits, 1)
                p_plan = _native.Plan(config, splits, 0)
                _, bn, _ = config_geometry(names[config])
                per = -(-kt.value // min(splits, kt.value))
                lim = token_limit(names[config])
                if lim is not None:  # weight streaming: any K range quantizes in the kernel
                    fits = True
                    if m > lim:  # refused: more tokens than the tile holds
                        assert lib.bfp8_workspace_bytes(ctypes.byref(p), in_plan) < 0
                        assert "tokens" in lib.bfp8_last_error().decode()
                        continue
                else:
                    fits = names[config].startswith("w") and per * bn * 128 <= 65536
                expect = p_plan if fits else q_plan
                assert lib.bfp8_workspace_bytes(ctypes.byref(p), in_plan) == \
                    lib.bfp8_workspace_bytes(ctypes.byref(p), expect)
    bad = _native.Plan(99, 1, 0)
    p = _native.GemmProblem(M=1, N=128, K=128)
    assert lib.bfp8_workspace_bytes(ctypes.byref(p), bad) < 0
    assert "config" in lib.bfp8_last_error().decode()


def _stream_k_parts(tiles, k_tiles, ctas):
    """Parts per tile when ctas CTAs take the K-block positions
    [W b / G, W (b + 1) / G) of the tiles' K blocks in sequence."""
    work = tiles * k_tiles
    g = max(1, min(ctas, work))
    starts = [b * work // g for b in range(g)]
    parts = [1] * tiles
    for s_ in starts:
        if s_ % k_tiles:
            parts[s_ // k_tiles] += 1
    return parts, min(k_tiles, -(-work // g))  # a unit never leaves its tile


@pytest.mark.parametrize("m, n, k, ctas", [(1, 24576, 4096, 148), (16, 4096, 12288, 148),
                                           (37, 392, 2064, 5), (37, 392, 2064, 1000), (1, 128, 128, 148),
                                           (8192, 24576, 4096, 148)])
def test_stream_k_plan_sizes(m, n, k, ctas):
    """Workspace and counters of a stream-K plan (splits = -CTAs): the most
    parts any tile is cut into, times the tiles' fp32 partial tiles."""
    lib = _native.capi()
    names = [lib.bfp8_config_name(i).decode() for i in range(lib.bfp8_num_configs())]
    p = _native.GemmProblem(M=m, N=n, K=k)
    for config, name in enumerate(names):
        bm, bn, _ = config_geometry(name)
        lim = token_limit(name)
        if lim is not None:
            # weight streaming: the tiles are the weight rows only (all
            # tokens in one tile); parts are [128 rows][M rounded up to 4] fp32
            plan = _native.Plan(config, -ctas, 0)
            if m > lim:
                assert lib.bfp8_workspace_bytes(ctypes.byref(p), plan) < 0
                continue
            tiles = -(-n // 128)
            parts, _ = _stream_k_parts(tiles, -(-k // 128), ctas)
            most = max(parts)
            expect_ws = 0 if most == 1 else most * tiles * 128 * ((m + 3) & ~3) * 4
            assert lib.bfp8_workspace_bytes(ctypes.byref(p), plan) == expect_ws
            assert lib.bfp8_counters_needed(ctypes.byref(p), plan) == (0 if most == 1 else tiles)
            # quantization in the kernel needs no front; the kernel + GEMM mode does
            assert lib.bfp8_workspace_bytes(ctypes.byref(p), _native.Plan(config, -ctas, 2)) == expect_ws
            assert lib.bfp8_workspace_bytes(ctypes.byref(p), _native.Plan(config, -ctas, 1)) > expect_ws
            continue
        if bm == 256:  # CTA pairs: no stream-K schedule, refused with a reason
            assert lib.bfp8_workspace_bytes(ctypes.byref(p), _native.Plan(config, -ctas, 0)) < 0
            assert "stream-K" in lib.bfp8_last_error().decode()
            continue
        rows, cols = (n, m) if name.startswith("w") else (m, n)
        tiles = -(-rows // 128) * -(-cols // bn)
        parts, longest = _stream_k_parts(tiles, -(-k // 128), ctas)
        plan = _native.Plan(config, -ctas, 0)
        most = max(parts)
        expect_ws = 0 if most == 1 else most * tiles * 128 * bn * 4
        assert lib.bfp8_workspace_bytes(ctypes.byref(p), plan) == expect_ws
        assert lib.bfp8_counters_needed(ctypes.byref(p), plan) == (0 if most == 1 else tiles)
        # in-GEMM quantization needs the longest unit to fit the resident operand
        fits = name.startswith("w") and longest * bn * 128 <= 65536
        in_plan = _native.Plan(config, -ctas, 2)
        front = lib.bfp8_workspace_bytes(ctypes.byref(p), _native.Plan(config, -ctas, 1)) - expect_ws
        assert front > 0
        assert lib.bfp8_workspace_bytes(ctypes.byref(p), in_plan) == expect_ws + (0 if fits else front)


def test_c_abi_rejects_bad_problems_without_launching():
    lib = _native.capi()
    p = _native.GemmProblem(M=4, N=256, K=200)  # K % 16 != 0
    assert lib.bfp8_launch_gemm(ctypes.byref(p), _native.Plan(0, 1, 0), None, None, None) == -1
    assert "K must be" in lib.bfp8_last_error().decode()
    p = _native.GemmProblem(M=4, N=256, K=256)
    assert lib.bfp8_launch_gemm(ctypes.byref(p), _native.Plan(0, 0, 0), None, None, None) == -1
    assert "splits" in lib.bfp8_last_error().decode()
    q = _native.QuantProblem(M=4, K=12)
    assert lib.bfp8_launch_quantize(ctypes.byref(q), None) == -1


def test_decode_linear_plans_quantize_ahead_of_the_streaming_kernel():
    """Up to 32 tokens the plan is a weight-streaming configuration; the
    fused (linear) plan puts the quantization kernel ahead of it at every M
    (the streaming kernel prefetches weights while the quantizer runs)."""
    lib = _native.capi()
    names = [lib.bfp8_config_name(i).decode() for i in range(lib.bfp8_num_configs())]
    for n, k in [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288)]:
        for m in [1, 2, 3, 4, 8, 16, 17, 32]:
            plan = lib.bfp8_choose_plan(m, n, k, 148)
            fplan = lib.bfp8_choose_fused_plan(m, n, k, 148)
            assert names[plan.config].startswith("w128d") and plan.fused == 0
            assert (fplan.config, fplan.splits, fplan.fused) == (plan.config, plan.splits, 1)
            bn = int(names[plan.config][len("w128d"):])
            assert bn >= m and (bn == 16 or bn // 2 < m)  # the smallest token tile that holds M


def test_producer_abi_rejects_bad_problems_without_launching():
    lib = _native.capi()
    fake = 1 << 20  # aligned non-null addresses: every check runs before any CUDA call
    r = _native.RmsNormQuantProblem(x=fake, ldx=208, weight=fake, q=fake, ldq=208, s=fake, s_m=1, s_k=4,
                                    M=4, H=208, variance_epsilon=1e-6, eps=1e-10)
    assert lib.bfp8_launch_rmsnorm_quant(ctypes.byref(r), None) == -1
    assert "multiple of 128" in lib.bfp8_last_error().decode()
    r.H, r.ldx, r.ldq = 32768, 32768, 32768
    assert lib.bfp8_launch_rmsnorm_quant(ctypes.byref(r), None) == -1
    assert "at most 16384" in lib.bfp8_last_error().decode()
    r.H, r.ldx, r.ldq, r.q, r.y = 256, 256, 256, None, None
    assert lib.bfp8_launch_rmsnorm_quant(ctypes.byref(r), None) == -1
    assert "nothing to write" in lib.bfp8_last_error().decode()
    r.q, r.x = fake, fake + 8  # x not 16-byte aligned
    assert lib.bfp8_launch_rmsnorm_quant(ctypes.byref(r), None) == -1
    assert "16-byte aligned" in lib.bfp8_last_error().decode()
    r.x, r.residual = fake, fake  # residual without residual_out
    assert lib.bfp8_launch_rmsnorm_quant(ctypes.byref(r), None) == -1
    assert "residual" in lib.bfp8_last_error().decode()
    m = _native.SiluMulQuantProblem(x=fake, ldx=400, q=fake, ldq=200, s=fake, s_m=1, s_k=4, M=4, I=200, eps=1e-10)
    assert lib.bfp8_launch_silu_mul_quant(ctypes.byref(m), None) == -1
    assert "multiple of 128" in lib.bfp8_last_error().decode()
    m.I, m.ldx, m.ldq = 256, 256, 256  # x must hold [gate | up] = 512 per row
    assert lib.bfp8_launch_silu_mul_quant(ctypes.byref(m), None) == -1
    assert "[M, 2I]" in lib.bfp8_last_error().decode()
    m.M = 0  # an empty batch is a no-op
    assert lib.bfp8_launch_silu_mul_quant(ctypes.byref(m), None) == 0


def test_torch_op_schemas_are_the_reference_ones():
    schemas = {s.name: str(s) for s in torch._C._jit_get_all_schemas() if s.name.startswith("blockfp8::")}
    assert "blockfp8::gemm(Tensor a, Tensor a_scales, Tensor b, Tensor b_scales, int config=-1, " \
           "int split_k=0) -> Tensor" in schemas.values()
    assert "blockfp8::gemm_bf16(Tensor x, Tensor b, Tensor b_scales, int config=-1, " \
           "int split_k=0, float eps=1e-10) -> Tensor" in schemas.values()
    assert "blockfp8::quantize(Tensor x, float eps=1e-10) -> (Tensor, Tensor)" in schemas.values()
    assert "blockfp8::linear(Tensor x, Tensor b, Tensor b_scales) -> Tensor" in schemas.values()
    assert "blockfp8::prefers_fused(int m, int n, int k) -> bool" in schemas.values()
    assert torch.ops.blockfp8.config_names().split(";") == blockfp8.configs()
    assert isinstance(torch.ops.blockfp8.prefers_fused(1, 6144, 4096), bool)


def test_fake_kernels_give_the_output_layouts():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(5, 256, dtype=torch.bfloat16)
        b = torch.empty(128, 256, dtype=FP8)
        sb = torch.empty(1, 2)
        q, s = torch.ops.blockfp8.quantize(x, 1e-10)
        assert q.shape == (5, 256) and q.dtype == FP8 and s.shape == (5, 2) and s.stride() == (1, 5)
        assert torch.ops.blockfp8.linear(x, b, sb).shape == (5, 128)
        assert torch.ops.blockfp8.gemm_bf16(x, b, sb, -1, 0, 1e-10).dtype == torch.bfloat16


def test_row_parallel_linear_resolves_the_linear_function():
    """row_parallel_linear calls the API's linear (the package's `gemm`
    attribute is the gemm function, not the submodule)."""
    import inspect
    from blockfp8_b200 import gemm as gemm_attr, sharding
    from blockfp8_b200.gemm import linear
    assert callable(gemm_attr) and not inspect.ismodule(gemm_attr)
    src = inspect.getsource(sharding.row_parallel_linear)
    assert "from .gemm import linear" in src and callable(linear)


def test_row_parallel_sizes_and_argument_checks():
    """bfp8_tp_tiles / bfp8_tp_partial_bytes follow the tile grid (a CTA
    pair's tile counts twice); bfp8_launch_gemm_tp rejects bad groups before
    touching a device."""
    lib = _native.capi()
    names = [lib.bfp8_config_name(i).decode() for i in range(lib.bfp8_num_configs())]
    for m, n in [(1, 4096), (300, 520), (8192, 24576)]:
        p = _native.GemmProblem(M=m, N=n, K=2048)
        for config, name in enumerate(names):
            bm, bn, _ = config_geometry(name)
            if token_limit(name) is not None:  # weight streaming: no row-parallel variant
                assert lib.bfp8_tp_tiles(ctypes.byref(p), _native.Plan(config, 1, 0)) < 0
                assert "row-parallel" in lib.bfp8_last_error().decode()
                continue
            rows, cols = (n, m) if name.startswith("w") else (m, n)
            tiles = -(-rows // bm) * -(-cols // bn) * (bm // 128)
            plan = _native.Plan(config, 1, 0)
            assert lib.bfp8_tp_tiles(ctypes.byref(p), plan) == tiles
            for world in (1, 2, 8):
                assert lib.bfp8_tp_partial_bytes(ctypes.byref(p), plan, world) == world * tiles * 128 * bn * 4
            assert lib.bfp8_tp_partial_bytes(ctypes.byref(p), plan, 9) < 0
    p = _native.GemmProblem(a=256, lda=512, b=512, ldb=512, sa=1024, sa_m=1, sa_k=16, sb=2048, sb_n=4, sb_k=1,
                            c=4096, ldc=256, M=16, N=256, K=512)
    plan = _native.Plan(0, 1, 0)

    def launch(**kw):
        tp = _native.TpGroup(world=kw.get("world", 2), rank=kw.get("rank", 1), wait=0)
        for q in range(8):
            tp.partials[q], tp.counters[q], tp.out[q] = 8192, 16384, 4096 + 65536 * q
        tp.out[1] = kw.get("own", 4096)
        rc = lib.bfp8_launch_gemm_tp(ctypes.byref(p), plan, None, None, ctypes.byref(tp), None)
        return rc, lib.bfp8_last_error().decode()

    assert launch(world=0)[0] == _native.BFP8_EINVAL and "1..8" in launch(world=0)[1]
    assert launch(world=9)[0] == _native.BFP8_EINVAL
    assert "rank" in launch(rank=2)[1]
    assert "out[rank]" in launch(own=8192)[1]
    assert "aligned" in launch(own=4100)[1]
    rc, msg = launch()  # a valid group: the first CUDA call fails here (no device)
    assert rc == _native.BFP8_ECUDA, msg


def test_plan_table_rows_are_layer_or_shard_shapes():
    """Every tuned row is a Qwen3-8B linear or one GPU's shard of it under
    tensor parallelism 2/4/8 (autotune --tp), with a valid plan."""
    from blockfp8_b200 import autotune

    shapes = set(autotune.LAYERS.values()) | set(autotune.tp_layers((2, 4, 8)).values())
    assert autotune.tp_layers((2,))["qkv/tp2"] == (3072, 4096)
    assert autotune.tp_layers((2,))["down/tp2"] == (4096, 6144)
    rows = autotune.read_table()
    lib = _native.capi()
    assert rows and all((n, k) in shapes for n, k, _ in rows)
    for (n, k, m), (config, splits) in rows.items():
        assert 0 <= config < lib.bfp8_num_configs() and splits != 0
        # exact rows are returned as tuned; up to 32 tokens the planner takes the
        # weight-streaming configurations, and the tuned rows serve the
        # row-parallel kernel (whose configurations are the tile ones)
        chosen = lib.bfp8_choose_tp_plan(m, n, k, 148, 0) if m <= 32 else lib.bfp8_choose_plan(m, n, k, 148)
        assert chosen.config == config or m >= 256


def test_untabulated_decode_shapes_take_swapped_configurations():
    """The planner's fallback (no tuned row for the shape) keeps to the
    swapped decode configurations up to 32 tokens, as the tuned shapes do."""
    lib = _native.capi()
    names = [lib.bfp8_config_name(i).decode() for i in range(lib.bfp8_num_configs())]
    for n, k in [(3200, 4096), (5120, 5120), (13824, 5120), (392, 1152)]:
        for m in (1, 5, 16, 32):
            plan = lib.bfp8_choose_plan(m, n, k, 148)
            assert names[plan.config].startswith("w"), (n, k, m, names[plan.config])
