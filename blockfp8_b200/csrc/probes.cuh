// Roofline probes, measured on the GPU the kernels run on, in the same
// process: the dense e4m3 tensor-core rate (back-to-back
// tcgen05.mma.kind::f8f6f4 from shared memory, one CTA per SM, no operand
// traffic) and the HBM read rate (a streaming read of a caller buffer larger
// than L2).  They bound what the GEMM's two regimes can reach on this part.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

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

}  // namespace bfp8
