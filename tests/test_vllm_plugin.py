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
