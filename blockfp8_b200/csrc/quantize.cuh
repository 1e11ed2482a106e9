// Per-token 1 x 128 activation quantizer, bf16 -> float8_e4m3fn + float32
// scales.  Same arithmetic as the reference (blockfp8 csrc/quant_sm89.cu:
// 40-55, blockfp8/quant.py:25-64): amax over the group starting from eps,
// scale = amax / 448 (IEEE division), q = e4m3(clamp(x / scale, -448, 448))
// with round-to-nearest-even and saturation.  The code is this project's own.
//
// HBM-bound single pass.  A half-warp owns one row segment of kGroups
// consecutive 128-wide groups (kGroups x 256 contiguous bytes of bf16): each
// lane issues all kGroups 16-byte loads before using any, so enough bytes are
// in flight to cover the DRAM latency, then reduces each group's amax with a
// 4-step shuffle over the 16 lanes.  The 16 half-warps of a CTA take 16
// consecutive rows of the same group range, so with the M-major scale layout
// a CTA's scale stores for one group are 16 consecutive words.  Grid-stride
// over (row block, group block) tasks with a device-filling grid.
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
constexpr int kQuantRows = kQuantThreads / 16;  // rows per CTA task
constexpr int kQuantGroups = 4;                 // groups per half-warp task

__global__ void __launch_bounds__(kQuantThreads) quantize_kernel(const QuantParams p) {
  // A GEMM launched behind this kernel with programmatic dependent launch may
  // start now: it only reads our output after griddepcontrol.wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane16 = threadIdx.x & 15;
  const int half = threadIdx.x >> 4;  // 0 .. 15: the row within the task
  const int row_blocks = (p.M + kQuantRows - 1) / kQuantRows;
  const int group_blocks = (p.kb + kQuantGroups - 1) / kQuantGroups;
  const int64_t tasks = int64_t(row_blocks) * group_blocks;
#pragma unroll 1
  for (int64_t t = blockIdx.x; t < tasks; t += gridDim.x) {
    // Row blocks vary fastest: neighbouring CTAs share a group range, so
    // their scale stores land in the same lines.
    const int rb = int(t % row_blocks), gb = int(t / row_blocks);
    const int row = rb * kQuantRows + half;
    const bool row_ok = row < p.M;  // uniform per half-warp
    const __nv_bfloat16* xr = p.x + int64_t(row_ok ? row : 0) * p.ldx;

    uint4 v[kQuantGroups];
#pragma unroll
    for (int j = 0; j < kQuantGroups; ++j) {
      const int col = (gb * kQuantGroups + j) * 128 + lane16 * 8;
      v[j] = make_uint4(0u, 0u, 0u, 0u);  // zeros leave the amax alone
      if (row_ok && col < p.K) v[j] = __ldcs(reinterpret_cast<const uint4*>(xr + col));
    }
#pragma unroll
    for (int j = 0; j < kQuantGroups; ++j) {
      const int g = gb * kQuantGroups + j;
      const int col = g * 128 + lane16 * 8;
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[j]);
      float f[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 u = __bfloat1622float2(h[e]);
        f[2 * e] = u.x;
        f[2 * e + 1] = u.y;
      }
      float amax = p.eps;
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
      // All 32 lanes take part; the xor offsets stay inside each half-warp.
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float scale = amax / 448.f;
      if (row_ok && col < p.K) {
        uint32_t packed[2] = {0u, 0u};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 u = make_float2(fminf(fmaxf(f[2 * e] / scale, -448.f), 448.f),
                                       fminf(fmaxf(f[2 * e + 1] / scale, -448.f), 448.f));
          const uint32_t pair = __nv_cvt_float2_to_fp8x2(u, __NV_SATFINITE, __NV_E4M3);
          packed[e >> 1] |= pair << (16 * (e & 1));
        }
        *reinterpret_cast<uint2*>(p.q + int64_t(row) * p.ldq + col) = make_uint2(packed[0], packed[1]);
      }
      if (row_ok && g < p.kb && lane16 == 0) p.s[int64_t(row) * p.s_m + int64_t(g) * p.s_k] = scale;
    }
  }
}

}  // namespace bfp8
