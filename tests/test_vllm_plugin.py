"""The vLLM plugin: registration order and idempotence, the entry point, and
(on a B200) vLLM's own selection plus layer == blockfp8.linear + bias.
Restates the reference's tests/test_vllm_plugin.py for sm_100."""

import os

import pytest
import torch

pytest.importorskip("vllm")

import blockfp8  # noqa: E402
import blockfp8_vllm  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _candidates():
    from vllm.model_executor.kernels.linear import _POSSIBLE_FP8_BLOCK_KERNELS
    from vllm.platforms import PlatformEnum

    return [k.__name__ for k in _POSSIBLE_FP8_BLOCK_KERNELS[PlatformEnum.CUDA]]


def test_register_is_idempotent_and_goes_ahead_of_every_sm100_candidate():
    blockfp8_vllm.register()
    blockfp8_vllm.register()
    names = _candidates()
    assert names.count("BlockFp8LinearKernel") == 1
    mine = names.index("BlockFp8LinearKernel")
    for other in ("FlashInferFp8DeepGEMMDynamicBlockScaledKernel", "DeepGemmFp8BlockScaledMMKernel",
                  "CutlassFp8BlockScaledMMKernel", "MarlinFP8ScaledMMLinearKernel"):
        if other in names:
            assert mine < names.index(other), other


def test_entry_point_is_declared():
    text = open(os.path.join(ROOT, "pyproject.toml")).read()
    assert '[project.entry-points."vllm.general_plugins"]' in text
    assert 'blockfp8 = "blockfp8_vllm:register"' in text


def test_is_supported_only_on_sm100():
    from blockfp8_vllm.kernel import BlockFp8LinearKernel
    ok, reason = BlockFp8LinearKernel.is_supported(89)
    assert not ok
    if torch.cuda.is_available():
        return
    ok, reason = BlockFp8LinearKernel.is_supported(100)
    assert not ok and "CUDA" in reason  # no CUDA platform in this container


def test_scale_attribute_lookup_is_version_tolerant():
    from blockfp8_vllm.kernel import block_scale_of

    class P:
        pass

    for name in ("weight_scale_inv", "weight_scale", "block_scale"):
        p = P()
        setattr(p, name, torch.ones(1))
        assert block_scale_of(p) is getattr(p, name)


def _kernel(n, k):
    from vllm.config import VllmConfig, set_current_vllm_config
    from vllm.model_executor.kernels.linear import init_fp8_linear_kernel
    from vllm.model_executor.layers.quantization.utils.quant_utils import (
        GroupShape,
        create_fp8_quant_key,
    )

    blockfp8_vllm.register()
    with set_current_vllm_config(VllmConfig()):
        return init_fp8_linear_kernel(
            activation_quant_key=create_fp8_quant_key(static=False, group_shape=GroupShape(1, 128)),
            weight_quant_key=create_fp8_quant_key(static=True, group_shape=GroupShape(128, 128)),
            input_dtype=torch.bfloat16, out_dtype=torch.bfloat16, weight_shape=(n, k))


@pytest.mark.gpu
@pytest.mark.parametrize("m", [1, 16, 300])
def test_vllm_selects_it_and_the_layer_equals_blockfp8_linear(m):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    assert blockfp8.native_available()
    if torch.cuda.get_device_capability() != (10, 0):
        pytest.skip("the plugin only takes over on sm_100")
    from vllm.config import VllmConfig, set_current_vllm_config

    n, k = 1024, 2048
    kernel = _kernel(n, k)
    assert type(kernel).__name__ == "BlockFp8LinearKernel"
    g = torch.Generator(device="cuda").manual_seed(m)
    w, ws = blockfp8.quantize_weights(torch.randn(n, k, generator=g, device="cuda") * 0.02)
    layer = torch.nn.Module()
    layer.weight = torch.nn.Parameter(w.clone(), requires_grad=False)
    layer.weight_scale_inv = torch.nn.Parameter(ws.clone(), requires_grad=False)
    layer.input_scale = None
    with set_current_vllm_config(VllmConfig()):
        kernel.process_weights_after_loading(layer)
        x = torch.randn(2, m, k, generator=g, device="cuda").to(torch.bfloat16)
        bias = torch.randn(n, generator=g, device="cuda").to(torch.bfloat16)
        out = kernel.apply_weights(layer, x, bias)
    expect = blockfp8.linear(x.reshape(-1, k), w, ws) + bias
    assert out.shape == (2, m, n) and torch.equal(out.reshape(-1, n), expect)


# ---- the end-to-end driver's helpers (blockfp8_vllm/e2e.py), on CPU ----------------------

def test_e2e_model_dir_is_the_qwen3_8b_architecture(tmp_path):
    from transformers import AutoConfig

    from blockfp8_vllm import e2e

    cfg = AutoConfig.from_pretrained(e2e.write_model_dir(str(tmp_path / "m")))
    assert cfg.model_type == "qwen3"
    assert (cfg.num_hidden_layers, cfg.hidden_size, cfg.intermediate_size) == (36, 4096, 12288)
    assert (cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.vocab_size) == (32, 8, 128, 151936)
    q = cfg.quantization_config
    assert q["quant_method"] == "fp8" and q["activation_scheme"] == "dynamic" and q["weight_block_size"] == [128, 128]


def test_e2e_entry_points_are_discoverable(tmp_path):
    import importlib.metadata as md

    from blockfp8_vllm import e2e

    site = e2e.write_entry_points(str(tmp_path / "site"))
    eps = {ep.name: ep.value for d in md.distributions(path=[site])
           for ep in d.entry_points if ep.group == "vllm.general_plugins"}
    assert eps == e2e.ENTRY_POINTS
    assert eps["blockfp8"] == 'blockfp8_vllm:register'  # the entry point pyproject.toml declares


def test_e2e_weight_init_draws_block_fp8_weights():
    from blockfp8_vllm import e2e

    lin = torch.nn.Module()
    lin.weight = torch.nn.Parameter(torch.zeros(384, 512).to(blockfp8.FP8_DTYPE), requires_grad=False)
    lin.weight_scale_inv = torch.nn.Parameter(torch.zeros(3, 4), requires_grad=False)
    assert e2e.init_module_weights(lin) == 2
    w = blockfp8.dequantize_weights(lin.weight, lin.weight_scale_inv)
    assert abs(w.std().item() - e2e.WEIGHT_STD) < 0.05 * e2e.WEIGHT_STD
    wq, ws = blockfp8.quantize_weights(w)  # already on the e4m3 grid of its own block scales
    assert torch.equal(ws, lin.weight_scale_inv) and torch.equal(wq.view(torch.uint8), lin.weight.view(torch.uint8))

    norm, emb = torch.nn.Module(), torch.nn.Module()
    norm.weight = torch.nn.Parameter(torch.zeros(64, dtype=torch.bfloat16), requires_grad=False)
    emb.weight = torch.nn.Parameter(torch.zeros(1000, 64, dtype=torch.bfloat16), requires_grad=False)
    assert e2e.init_module_weights(norm) == 1 and torch.all(norm.weight == 1)
    assert e2e.init_module_weights(emb) == 1 and abs(emb.weight.float().std().item() - 0.02) < 0.002

    bad = torch.nn.Module()
    bad.weight = torch.nn.Parameter(torch.zeros(256, 256).to(blockfp8.FP8_DTYPE), requires_grad=False)
    bad.weight_scale_inv = torch.nn.Parameter(torch.zeros(1, 1), requires_grad=False)
    with pytest.raises(RuntimeError, match="block scales"):
        e2e.init_module_weights(bad)


def test_e2e_weight_init_wraps_the_dummy_loader_once(monkeypatch):
    from vllm.model_executor.model_loader import dummy_loader

    from blockfp8_vllm import e2e

    monkeypatch.setattr(dummy_loader, "initialize_dummy_weights", dummy_loader.initialize_dummy_weights)
    e2e.install_weight_init()
    patched = dummy_loader.initialize_dummy_weights
    e2e.install_weight_init()
    assert dummy_loader.initialize_dummy_weights is patched and patched.blockfp8_e2e

    parent, child = torch.nn.Module(), torch.nn.Module()
    child.weight = torch.nn.Parameter(torch.zeros(256, 128).to(blockfp8.FP8_DTYPE), requires_grad=False)
    child.weight_scale_inv = torch.nn.Parameter(torch.zeros(2, 1), requires_grad=False)
    parent.child = child
    for m in parent.modules():  # the loader's order: parents first
        patched(m, None)
    assert torch.all(child.weight_scale_inv > 0)
    assert blockfp8.dequantize_weights(child.weight, child.weight_scale_inv).abs().max() > 0.02


def test_e2e_agreement_summary():
    from blockfp8_vllm import e2e

    stock = {"greedy": [{"tokens": [1, 2, 3], "logprobs": [-1.0, -2.0, -3.0]},
                        {"tokens": [4, 5], "logprobs": [-0.5, -0.5]}]}
    plugin = {"greedy": [{"tokens": [1, 2, 9]}, {"tokens": [4, 5]}],
              "teacher_forced": [[-1.0, -2.5, -3.0], [-0.5, -0.25]]}
    a = e2e.compare(stock, plugin)
    assert a["greedy_tokens_agreeing"] == [2, 2]
    assert a["teacher_forced_logprob_abs_diff_max"] == 0.5
    assert abs(a["teacher_forced_logprob_abs_diff_mean"] - 0.75 / 5) < 1e-12
