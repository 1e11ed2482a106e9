// Roofline probes, measured on the GPU the kernels run on, in the same
// process: the dense e4m3 tensor-core rate (back-to-back
// tcgen05.mma.kind::f8f6f4 from shared memory, one CTA per SM, no operand
// traffic) and the HBM read rate (a streaming read of a caller buffer larger
// than L2).  They bound what the GEMM's two regimes can reach on this part.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"
#include "quant_math.cuh"

namespace bfp8 {

constexpr uint32_t kProbeWaitSite = 9;  // status site of the probe's bounded wait

// 128 x N x 32 e4m3 MMAs into one TMEM buffer, `iters` groups of four, from
// zeroed operand tiles; the CTA's elapsed clocks go to
// clocks[blockIdx.x].  Shared memory is sized so one CTA fits on an SM (each
// allocates all of TMEM).
template <int N>
__global__ void __launch_bounds__(128, 1) probe_mma_kernel(int iters, unsigned long long* clocks) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  __shared__ uint64_t done;
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (128 + N) * 128 / 16; i += blockDim.x)
    st_shared_v4(base + uint32_t(i) * 16u, 0u, 0u, 0u, 0u);
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&done), 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&slot), 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot;
  if (threadIdx.x == 0) {
    const uint64_t da = smem_desc_k128_sw128(base), db = smem_desc_k128_sw128(base + 128 * 128);
    constexpr uint32_t idesc = idesc_e4m3_f32(128, N);
    const long long t0 = clock64();
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int k = 0; k < 4; ++k) mma_f8(tmem, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
    mma_commit(smem_u32(&done));
    mbar_wait(smem_u32(&done), 0, nullptr, kProbeWaitSite);
    clocks[blockIdx.x] = static_cast<unsigned long long>(clock64() - t0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// One 128 x 32 x 128 block product exactly as the GEMM forms a K block's
// partial: A [128 x 128] and B [32 x 128] e4m3 (row-major, 128 bytes a row)
// into 128-byte-swizzled shared memory, four K = 32 MMAs into TMEM (the
// first with the accumulator input off), and the raw fp32 result
// D [128 x 32] back to global memory.  For precision experiments.
__global__ void __launch_bounds__(128, 1) probe_block_kernel(const uint8_t* __restrict__ a,
                                                             const uint8_t* __restrict__ b, float* d) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sb_tile = base + 128 * 128;
  __shared__ uint64_t done;
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5, row = threadIdx.x;
  // 16-byte unit u of row r sits at r * 128 + ((u ^ (r % 8)) * 16)
  for (int u = 0; u < 8; ++u) {
    const uint4 v = reinterpret_cast<const uint4*>(a + row * 128)[u];
    st_shared_v4(base + uint32_t(row) * 128u + uint32_t((u ^ (row & 7)) * 16), v.x, v.y, v.z, v.w);
    if (row < 32) {
      const uint4 w = reinterpret_cast<const uint4*>(b + row * 128)[u];
      st_shared_v4(sb_tile + uint32_t(row) * 128u + uint32_t((u ^ (row & 7)) * 16), w.x, w.y, w.z, w.w);
    }
  }
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&done), 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&slot), 32);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot;
  if (threadIdx.x == 0) {
    const uint64_t da = smem_desc_k128_sw128(base), db = smem_desc_k128_sw128(sb_tile);
    constexpr uint32_t idesc = idesc_e4m3_f32(128, 32);
#pragma unroll
    for (int k = 0; k < 4; ++k) mma_f8(tmem, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
    mma_commit(smem_u32(&done));
  }
  mbar_wait(smem_u32(&done), 0, nullptr, kProbeWaitSite);
  tc_fence_after();
  float v[32];
  tmem_ld32(tmem + (uint32_t(32 * warp) << 16), v);
#pragma unroll
  for (int j = 0; j < 32; ++j) d[row * 32 + j] = v[j];
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

// Reads every 16-byte word of buf once (grid-stride); one xor per thread goes
// to sink so the loads are not dead.
__global__ void __launch_bounds__(256) probe_read_kernel(const uint4* __restrict__ buf, int64_t words,
                                                         uint32_t* sink) {
  uint32_t acc = 0;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < words; i += 4 * stride) {  // four loads in flight per thread
    const uint4 a = __ldcs(buf + i), b = __ldcs(buf + i + stride), c = __ldcs(buf + i + 2 * stride),
                d = __ldcs(buf + i + 3 * stride);
    acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
  }
  for (; i < words; i += stride) {
    const uint4 a = __ldcs(buf + i);
    acc ^= a.x ^ a.y ^ a.z ^ a.w;
  }
  sink[blockIdx.x * blockDim.x + threadIdx.x] = acc;
}

// Exhaustive check of the quantizer's fast path (group_codes_fast) against
// the reference's sequence (group_codes_exact) on its whole input domain:
// block a uses amax = max(eps, the bf16 magnitude with bits a), a in
// [0, 0x7F80) (a = 0 gives amax = eps), and its threads cover all 65536 bf16
// patterns x, 8 at a time; x that is not finite or above amax cannot occur
// in a group with that amax and is skipped.  out[0] counts the codes that
// differ, out[1] holds the first mismatch as (a << 32) | x + 1.
__global__ void __launch_bounds__(256) probe_quant_kernel(float eps, unsigned long long* out) {
  const uint32_t a = blockIdx.x;
  const float amax = fmaxf(eps, __uint_as_float(a << 16));
  const float scale = amax / 448.f;  // the reference's division
  const float r = __frcp_rn(scale);
  unsigned long long bad = 0;
  for (uint32_t x0 = threadIdx.x * 8u; x0 < 65536u; x0 += blockDim.x * 8u) {
    const uint4 v = make_uint4(x0 | ((x0 + 1u) << 16), (x0 + 2u) | ((x0 + 3u) << 16), (x0 + 4u) | ((x0 + 5u) << 16),
                               (x0 + 6u) | ((x0 + 7u) << 16));
    float f[8];
    bf16x8_to_float(v, f);
    const uint2 fast = group_codes_fast(v, scale, r);
    const uint2 exact = group_codes_exact(f, scale);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t x = x0 + uint32_t(e);
      const bool valid = (x & 0x7FFFu) < 0x7F80u && fabsf(f[e]) <= amax;
      const uint32_t cf = ((e < 4 ? fast.x : fast.y) >> (8 * (e & 3))) & 0xFFu;
      const uint32_t ce = ((e < 4 ? exact.x : exact.y) >> (8 * (e & 3))) & 0xFFu;
      if (valid && cf != ce) {
        ++bad;
        atomicCAS(out + 1, 0ull, (static_cast<unsigned long long>(a) << 32) | (x + 1u));
      }
    }
  }
  if (bad) atomicAdd(out, bad);
}

// scale_of (the quantizer's three-operation amax / 448) against the IEEE
// division on every finite non-negative float: thread i of the grid checks
// bit patterns i, i + stride, ... below 0x7F800000.  out[0] counts the
// differences, out[1] holds the first as its bit pattern + 1.
__global__ void __launch_bounds__(256) probe_scale_kernel(unsigned long long* out) {
  unsigned long long bad = 0;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t b = blockIdx.x * blockDim.x + threadIdx.x; b < 0x7F800000u; b += stride) {
    const float a = __uint_as_float(b);
    if (__float_as_uint(scale_of(a)) != __float_as_uint(a / 448.f)) {
      ++bad;
      atomicCAS(out + 1, 0ull, static_cast<unsigned long long>(b) + 1ull);
    }
  }
  if (bad) atomicAdd(out, bad);
}

}  // namespace bfp8
