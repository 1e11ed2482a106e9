// Per-token 1 x 128 activation quantizer, bf16 -> float8_e4m3fn + float32
// scales.  Same arithmetic as the reference (blockfp8 csrc/quant_sm89.cu:
// 40-55, blockfp8/quant.py:25-64): amax over the group starting from eps,
// scale = amax / 448 (IEEE division), q = e4m3(clamp(x / scale, -448, 448))
// with round-to-nearest-even and saturation.  The code is this project's own.
//
// HBM-bound single pass: 16 lanes per 128-wide group, one 16-byte load and
// one 8-byte store per lane, a 4-step shuffle for the group amax.  Groups
// are numbered row-fastest (g = kb * M + row), so with the M-major scale
// layout the scale stores of neighbouring groups are neighbouring words, and
// a CTA reads 16 rows' worth of one 256-byte K slice per step.  Grid-stride
// over groups with a device-filling grid.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdint>

namespace bfp8 {

struct QuantParams {
  const __nv_bfloat16* x;
  int64_t ldx;
  uint8_t* q;
  int64_t ldq;
  float* s;
  int64_t s_m, s_k;
  int M, K, kb;
  float eps;
};

constexpr int kQuantThreads = 256;

__global__ void __launch_bounds__(kQuantThreads) quantize_kernel(const QuantParams p) {
  const int lane16 = threadIdx.x & 15;
  const int64_t groups = int64_t(p.M) * p.kb;
  // Both halves of a warp iterate together (the shuffle below needs all 32
  // lanes); a half past the end carries zeros and stores nothing.
  const int64_t warp_first = (int64_t(blockIdx.x) * kQuantThreads + (threadIdx.x & ~31)) / 16;
  const int64_t stride = int64_t(gridDim.x) * (kQuantThreads / 16);
#pragma unroll 1
  for (int64_t g0 = warp_first; g0 < groups; g0 += stride) {
    const int64_t g = g0 + ((threadIdx.x >> 4) & 1);
    const bool valid = g < groups;
    const int64_t row = valid ? g % p.M : 0;
    const int kbi = valid ? int(g / p.M) : 0;
    const int col = kbi * 128 + lane16 * 8;
    const bool in = valid && col < p.K;  // K % 8 == 0: a lane's 8 values are all in or all out

    uint4 v = make_uint4(0u, 0u, 0u, 0u);  // zeros leave the amax alone
    if (in) v = __ldcs(reinterpret_cast<const uint4*>(p.x + row * p.ldx + col));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
    float f[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = __bfloat1622float2(h[e]);
      f[2 * e] = t.x;
      f[2 * e + 1] = t.y;
    }
    float amax = p.eps;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = amax / 448.f;

    if (in) {
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 t = make_float2(fminf(fmaxf(f[2 * e] / scale, -448.f), 448.f),
                                     fminf(fmaxf(f[2 * e + 1] / scale, -448.f), 448.f));
        const uint32_t pair = __nv_cvt_float2_to_fp8x2(t, __NV_SATFINITE, __NV_E4M3);
        packed[e >> 1] |= pair << (16 * (e & 1));
      }
      *reinterpret_cast<uint2*>(p.q + row * p.ldq + col) = make_uint2(packed[0], packed[1]);
    }
    if (valid && lane16 == 0) p.s[row * p.s_m + int64_t(kbi) * p.s_k] = scale;
  }
}

}  // namespace bfp8
