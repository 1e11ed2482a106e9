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

#include "quant_math.cuh"

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
constexpr int kQuantGroups = 4;                 // groups per half-warp task (large batches)

// G groups per half-warp task: 4 for large batches (more bytes in flight per
// lane), 1 for decode-sized ones, whose few row blocks would otherwise leave
// most SMs idle while each half-warp quantizes four groups one after another.
template <int G>
__global__ void __launch_bounds__(kQuantThreads) quantize_kernel(const QuantParams p) {
  // A GEMM launched behind this kernel with programmatic dependent launch may
  // start now: it only reads our output after griddepcontrol.wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // This kernel may itself start before the previous kernel of the stream
  // has finished: x may be its output, and q and s may still be read by it.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane16 = threadIdx.x & 15;
  const int half = threadIdx.x >> 4;  // 0 .. 15: the row within the task
  const int row_blocks = (p.M + kQuantRows - 1) / kQuantRows;
  const int group_blocks = (p.kb + G - 1) / G;
  const int tasks = row_blocks * group_blocks;  // < 2^31 (checked by the host)
  // Task t: rows rb * 16 .. + 15 (one per half-warp), groups gb * G .. + G - 1.
  // Row blocks vary fastest: neighbouring CTAs share a group range, so their
  // scale stores land in the same lines.  The loads of a CTA's next task go
  // out before the current one is converted.
  auto load = [&](int t, uint4 (&v)[G]) {
    const int gb = t / row_blocks, rb = t - gb * row_blocks;
    const int row = rb * kQuantRows + half;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int col = (gb * G + j) * 128 + lane16 * 8;
      v[j] = make_uint4(0u, 0u, 0u, 0u);  // zeros leave the amax alone
      if (row < p.M && col < p.K) v[j] = __ldcs(reinterpret_cast<const uint4*>(p.x + int64_t(row) * p.ldx + col));
    }
  };
  uint4 cur[G], nxt[G];
  int t = blockIdx.x;
  if (t < tasks) load(t, cur);
#pragma unroll 1
  for (; t < tasks; t += gridDim.x) {
    if (t + int(gridDim.x) < tasks) load(t + gridDim.x, nxt);
    const int gb = t / row_blocks, rb = t - gb * row_blocks;
    const int row = rb * kQuantRows + half;
    const bool row_ok = row < p.M;  // uniform per half-warp
    uint8_t* qrow = p.q + int64_t(row) * p.ldq;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int g = gb * G + j;
      const int col = g * 128 + lane16 * 8;
      const GroupQuant gq = quantize_group(cur[j], p.eps);  // all 32 lanes (shuffles)
      if (row_ok && col < p.K) *reinterpret_cast<uint2*>(qrow + col) = gq.codes;
      if (row_ok && g < p.kb && lane16 == 0) p.s[int64_t(row) * p.s_m + int64_t(g) * p.s_k] = gq.scale;
    }
#pragma unroll
    for (int j = 0; j < G; ++j) cur[j] = nxt[j];
  }
}

}  // namespace bfp8
