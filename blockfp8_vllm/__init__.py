"""vLLM plugin: run block-FP8 linear layers on B200 (sm_100) with blockfp8.linear.

register() is the `vllm.general_plugins` entry point (pyproject.toml:
blockfp8 = "blockfp8_vllm:register"), which vLLM calls in each of its
processes.  It puts BlockFp8LinearKernel at the head of vLLM's CUDA block-FP8
kernel list, ahead of every sm_100-capable candidate (FlashInfer/DeepGEMM,
DeepGEMM, CUTLASS).  vLLM takes the first candidate that reports itself
supported and able to implement a layer, so the kernel takes over exactly
where it applies (sm_100, bf16, 128x128 weight blocks, dynamic 1x128
activation groups) and every other GPU or layer keeps vLLM's own choice.
Nothing in the installed vLLM is edited.

Counterpart of the reference's blockfp8_vllm/__init__.py:24-42, which
inserted ahead of Marlin for sm_89; on B200 the competitors sit earlier in
the list, so the insertion point moves to the front.

To run stock vLLM with this package installed, leave "blockfp8" out of
VLLM_PLUGINS.
"""

import logging

logger = logging.getLogger(__name__)

_registered = False


def register() -> None:
    """Entry point; safe to call more than once per process."""
    global _registered
    if _registered:
        return
    from vllm.model_executor.kernels import linear as linear_kernels
    from vllm.platforms import PlatformEnum

    from .kernel import BlockFp8LinearKernel

    candidates = linear_kernels._POSSIBLE_FP8_BLOCK_KERNELS.setdefault(PlatformEnum.CUDA, [])
    if BlockFp8LinearKernel not in candidates:
        ahead_of = candidates[0].__name__ if candidates else "nothing"
        candidates.insert(0, BlockFp8LinearKernel)
        logger.info("blockfp8: BlockFp8LinearKernel inserted ahead of %s", ahead_of)
    _registered = True
