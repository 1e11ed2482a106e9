"""Tensor layouts of the block-FP8 linear path (DeepSeek-V3 / Qwen3-FP8 style).

  activations  A_q      [M, K]            float8_e4m3fn, row-major (K contiguous)
               A_scales [M, ceil(K/128)]  float32, one per row per 128-wide K
                                          group; any strides (the quantizer
                                          writes M-contiguous ones, (1, M))
  weights      B_q      [N, K]            float8_e4m3fn, row-major ("weight")
               B_scales [ceil(N/128), ceil(K/128)]  float32, one per 128 x 128
                                          block ("weight_scale_inv")
  output       C        [M, N]            bfloat16, row-major

  C[m, n] = sum_kb A_scales[m, kb] * B_scales[n // 128, kb]
                   * sum_{k in block kb} A_q[m, k] * B_q[n, k]

The scales multiply (w = w_q * scale), whatever the checkpoint calls them.
Same contract as the reference (simon-jd/blockfp8 blockfp8/layout.py:1-35).
"""

import torch

FP8_DTYPE = torch.float8_e4m3fn
FP8_MAX = 448.0  # largest finite float8_e4m3fn
GROUP_K = 128  # activation group width and weight block width along K
BLOCK_N = 128  # weight block height along N

# TMA needs 16-byte rows of e4m3 along K; the op layer accepts N in steps of 8.
K_ALIGN = 16
N_ALIGN = 8


def cdiv(a: int, b: int) -> int:
    return -(-a // b)
