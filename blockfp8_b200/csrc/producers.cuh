// The layers that feed a block-FP8 linear, emitting its operand directly:
// RMSNorm (optionally after a residual add) and SiLU-and-mul, each followed by
// the activation quantizer's 1 x 128 e4m3 quantization in the same kernel.
// The linear after them then runs the GEMM alone -- no quantization launch
// and no bf16 round trip through HBM between the two.
//
// Arithmetic, per row (the usual decoder-layer definitions, as vLLM's
// RMSNorm and SiLU-and-mul compute them):
//   RMSNorm:  h = bf16(x + residual) when a residual is given, else x;
//             rstd = rsqrt(sum(h^2) / H + variance_epsilon) (fp32);
//             y = bf16(bf16(h * rstd) * weight)
//   SiLU-mul: g, u = x[:, :I], x[:, I:];  y = bf16(bf16(g / (1 + exp(-g))) * u)
// and then exactly the quantizer's mapping of y (quant_math.cuh): the codes
// and scales are those blockfp8.quantize_cuda gives for the bf16 y the kernel
// can also write out (tests compare them bit for bit).
//
// Layout: a thread owns 16 consecutive values (two 16-byte loads), so a
// 128-value group is 8 consecutive lanes and its amax is one warp reduction
// over those lanes.  RMSNorm: one CTA of 256 threads per row (the row sum is
// a block reduction), rows up to 16384 values held in registers.  SiLU-mul:
// CTAs over (row, 4096-column chunk), no reduction beyond the groups.  Both
// launch with programmatic dependent launch and wait (griddepcontrol.wait)
// before they read their inputs.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdint>

#include "ptx.cuh"
#include "quant_math.cuh"

namespace bfp8 {

constexpr int kProdThreads = 256;
constexpr int kProdChunk = kProdThreads * 16;  // values a CTA covers per pass
constexpr int kProdMaxChunks = 4;              // RMSNorm rows up to 16384 values

struct RmsNormQuantParams {
  const __nv_bfloat16* x;
  int64_t ldx;
  const __nv_bfloat16* residual;  // nullable
  int64_t ldr;
  __nv_bfloat16* residual_out;  // bf16(x + residual), written when residual is given
  int64_t ldro;
  const __nv_bfloat16* weight;  // [H]
  __nv_bfloat16* y;             // nullable: the normalized bf16 row
  int64_t ldy;
  uint8_t* q;  // nullable (then only y): e4m3 codes
  int64_t ldq;
  float* s;
  int64_t s_m, s_k;
  int M, H;
  float variance_epsilon, eps;
};

struct SiluMulQuantParams {
  const __nv_bfloat16* x;  // [M, 2I]: gate then up
  int64_t ldx;
  __nv_bfloat16* y;  // nullable: the bf16 product [M, I]
  int64_t ldy;
  uint8_t* q;  // nullable (then only y)
  int64_t ldq;
  float* s;
  int64_t s_m, s_k;
  int M, I;
  float eps;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // a -> low half
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Quantize the 16 bf16 values of this lane (v0: values 0-7, v1: 8-15), its
// group being 8 consecutive lanes (lanes 8k .. 8k + 7, all 32 lanes calling).
// Writes the 16 codes (16 bytes, may be null) and returns the group's scale.
__device__ __forceinline__ float quantize16(const uint4& v0, const uint4& v1, float eps, uint8_t* codes) {
  const uint32_t lane_mask = 0xFFu << (threadIdx.x & 24u);
  const uint32_t m0 = __vmaxu2(__vmaxu2(v0.x & 0x7FFF7FFFu, v0.y & 0x7FFF7FFFu),
                               __vmaxu2(v0.z & 0x7FFF7FFFu, v0.w & 0x7FFF7FFFu));
  const uint32_t m1 = __vmaxu2(__vmaxu2(v1.x & 0x7FFF7FFFu, v1.y & 0x7FFF7FFFu),
                               __vmaxu2(v1.z & 0x7FFF7FFFu, v1.w & 0x7FFF7FFFu));
  const uint32_t m2 = __vmaxu2(m0, m1);
  const uint32_t mbits = __reduce_max_sync(lane_mask, max(m2 & 0xFFFFu, m2 >> 16));
  float scale;
  uint2 c0, c1;
  if (mbits < 0x7F80u) {  // finite group (uniform over its 8 lanes)
    scale = scale_of(fmaxf(eps, __uint_as_float(mbits << 16)));
    const float r = __frcp_rn(scale);
    c0 = group_codes_fast(v0, scale, r);
    c1 = group_codes_fast(v1, scale, r);
  } else {  // an infinity or NaN: the reference's sequence (NaN dropped from the amax)
    float f0[8], f1[8];
    bf16x8_to_float(v0, f0);
    bf16x8_to_float(v1, f1);
    float amax = eps;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fmaxf(fabsf(f0[e]), fabsf(f1[e])));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(lane_mask, amax, o));
    scale = amax / 448.f;
    c0 = group_codes_exact(f0, scale);
    c1 = group_codes_exact(f1, scale);
  }
  if (codes) *reinterpret_cast<uint4*>(codes) = make_uint4(c0.x, c0.y, c1.x, c1.y);
  return scale;
}

__global__ void __launch_bounds__(kProdThreads) rmsnorm_quant_kernel(const RmsNormQuantParams p) {
  griddep_launch_dependents();
  griddep_wait();  // x and residual may be the previous kernel's output
  const int row = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int nchunks = (p.H + kProdChunk - 1) / kProdChunk;
  uint4 h[kProdMaxChunks][2];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kProdMaxChunks; ++c) {
    h[c][0] = h[c][1] = make_uint4(0u, 0u, 0u, 0u);
    const int col = c * kProdChunk + t * 16;
    if (c < nchunks && col < p.H) {
      const uint4* xs = reinterpret_cast<const uint4*>(p.x + int64_t(row) * p.ldx + col);
      h[c][0] = xs[0];
      h[c][1] = xs[1];
      if (p.residual) {
        const uint4* rs = reinterpret_cast<const uint4*>(p.residual + int64_t(row) * p.ldr + col);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint4 rv = rs[k];
          float a[8], b[8];
          bf16x8_to_float(h[c][k], a);
          bf16x8_to_float(rv, b);
          h[c][k] = make_uint4(pack_bf16x2(a[0] + b[0], a[1] + b[1]), pack_bf16x2(a[2] + b[2], a[3] + b[3]),
                               pack_bf16x2(a[4] + b[4], a[5] + b[5]), pack_bf16x2(a[6] + b[6], a[7] + b[7]));
        }
        uint4* ro = reinterpret_cast<uint4*>(p.residual_out + int64_t(row) * p.ldro + col);
        ro[0] = h[c][0];
        ro[1] = h[c][1];
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float a[8];
        bf16x8_to_float(h[c][k], a);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(a[e], a[e], ss);
      }
    }
  }
  // Row sum: warps, then the 8 warp sums in a fixed order.
  __shared__ float part[kProdThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kProdThreads / 32; ++w) tot += part[w];
  const float rstd = rsqrtf(tot / float(p.H) + p.variance_epsilon);
#pragma unroll
  for (int c = 0; c < kProdMaxChunks; ++c) {
    if (c >= nchunks) break;  // CTA-uniform
    const int col = c * kProdChunk + t * 16;
    const bool in = col < p.H;  // whole 8-lane groups (H % 128 == 0)
    uint4 y[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
    if (in) {
      const uint4* ws = reinterpret_cast<const uint4*>(p.weight + col);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float a[8], w[8], o[8];
        bf16x8_to_float(h[c][k], a);
        bf16x8_to_float(ws[k], w);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          o[e] = __bfloat162float(__float2bfloat16_rn(a[e] * rstd)) * w[e];  // bf16(h rstd) * weight
        y[k] = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                          pack_bf16x2(o[6], o[7]));
      }
      if (p.y) {
        uint4* yo = reinterpret_cast<uint4*>(p.y + int64_t(row) * p.ldy + col);
        yo[0] = y[0];
        yo[1] = y[1];
      }
    }
    if (p.q) {
      const float scale = quantize16(y[0], y[1], p.eps, in ? p.q + int64_t(row) * p.ldq + col : nullptr);
      if (in && (lane & 7) == 0) p.s[int64_t(row) * p.s_m + int64_t(col / 128) * p.s_k] = scale;
    }
  }
}

__global__ void __launch_bounds__(kProdThreads) silu_mul_quant_kernel(const SiluMulQuantParams p) {
  griddep_launch_dependents();
  griddep_wait();  // x may be the previous kernel's output
  const int row = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int col = blockIdx.x * kProdChunk + threadIdx.x * 16;
  const bool in = col < p.I;  // whole 8-lane groups (I % 128 == 0)
  uint4 y[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
  if (in) {
    const uint4* gs = reinterpret_cast<const uint4*>(p.x + int64_t(row) * p.ldx + col);
    const uint4* us = reinterpret_cast<const uint4*>(p.x + int64_t(row) * p.ldx + p.I + col);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float g[8], u[8], o[8];
      bf16x8_to_float(gs[k], g);
      bf16x8_to_float(us[k], u);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        o[e] = __bfloat162float(__float2bfloat16_rn(g[e] / (1.f + expf(-g[e])))) * u[e];
      y[k] = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]),
                        pack_bf16x2(o[6], o[7]));
    }
    if (p.y) {
      uint4* yo = reinterpret_cast<uint4*>(p.y + int64_t(row) * p.ldy + col);
      yo[0] = y[0];
      yo[1] = y[1];
    }
  }
  if (p.q) {
    const float scale = quantize16(y[0], y[1], p.eps, in ? p.q + int64_t(row) * p.ldq + col : nullptr);
    if (in && (lane & 7) == 0) p.s[int64_t(row) * p.s_m + int64_t(col / 128) * p.s_k] = scale;
  }
}

}  // namespace bfp8
