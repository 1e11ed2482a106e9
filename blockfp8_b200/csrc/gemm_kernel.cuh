// Block-scaled FP8 GEMM for sm_100a (B200):
//
//   C[m, n] = sum_kb sa[m, kb] * sb[n / 128, kb] * sum_{k in kb} A[m, k] * B[n, k]
//
// One persistent, warp-specialised CTA per SM walks a static list of work
// units (an output tile of 128 x BN and a range of 128-wide K blocks):
//
//   warp 0      TMA producer: A tile [128 x 128 B] and B tile [BN x 128 B]
//               of each K block into a STAGES-deep shared-memory ring
//               (128-byte swizzle), completion counted in bytes on the
//               stage's "full" mbarrier;
//   warp 1      MMA issuer (one thread): per K block, four
//               tcgen05.mma.kind::f8f6f4 (K = 32 each, e4m3 x e4m3 -> f32)
//               into one of ACC_BUFS tensor-memory (TMEM) partial buffers,
//               the first with the accumulator input disabled, so the buffer
//               holds exactly that block's unscaled partial sums; then
//               tcgen05.commit frees the smem stage and publishes the buffer;
//   warps 2..   promotion + epilogue (EPI_WG warpgroups; warp w reads TMEM
//               lanes 32 * (w % 4) ..): tcgen05.ld the partial, multiply by
//               sa[m, kb] * sb[nb, kb] and add into fp32 registers with one
//               fmaf per value (the promotion of the reference kernel,
//               blockfp8 csrc/gemm_kernel.cuh:372-382, same operation
//               order), release the buffer; after the unit's last K block,
//               round to bf16 into a swizzled smem tile and TMA-store it.
//
// Because every K block gets its own TMEM buffer, the MMAs of block k + 1
// run while block k is being promoted.  With split-K the units of one tile
// cover disjoint K ranges; each writes its fp32 partial tile to a workspace
// and the last to arrive (an atomic counter) sums the partials in split order
// 0, 1, ..., S - 1 and stores the tile, as the reference does
// (blockfp8 csrc/gemm_kernel.cuh:403-448), so results are deterministic and
// no CTA ever waits for another.
//
// Every mbarrier wait is bounded (ptx.cuh): on a timeout the kernel records a
// status code, drains its in-flight copies and MMAs, frees TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdint>

#include "ptx.cuh"

namespace bfp8 {

struct GemmParams {
  CUtensorMap map_a;  // A e4m3 [M, K] (row stride lda), box 128 x 128, 128B swizzle
  CUtensorMap map_b;  // B e4m3 [N, K] (row stride ldb), box 128 x BN, 128B swizzle
  CUtensorMap map_c;  // C bf16 [M, N] (row stride ldc), box 64 x 32, 128B swizzle
  const float* sa;
  int64_t sa_m, sa_k;
  const float* sb;
  int64_t sb_n, sb_k;
  float* workspace;  // split-K partial tiles: [splits][tiles][128][BN] fp32
  int* counters;     // split-K arrivals, one per tile, zero between launches
  int M, N, K;
  int tiles_m, tiles_n, tiles;
  int k_tiles, k_per_split, splits;
  int units;  // tiles * splits
  int group_m;
  int stream_b;  // 1: B is read once (decode), hint L2 to evict it first
};

template <int BN_, int STAGES_>
struct GemmCfg {
  static constexpr int BM = 128, BN = BN_, BK = 128, STAGES = STAGES_;
  static_assert(BN == 64 || BN == 128 || BN == 256, "MMA N of 64, 128 or 256");
  static constexpr int COLS = BN < 128 ? BN : 128;  // accumulators per epilogue thread
  static constexpr int EPI_WG = BN / COLS;
  static constexpr int EPI_WARPS = 4 * EPI_WG;
  static constexpr int EPI_THREADS = 32 * EPI_WARPS;
  static constexpr int THREADS = 64 + EPI_THREADS;
  static constexpr int ACC_BUFS = 512 / BN > 4 ? 4 : 512 / BN;
  static constexpr int TMEM_COLS = ACC_BUFS * BN;  // 256 or 512: a power of two >= 32
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int OUT_BYTES = 32 * 128;  // per epilogue warp: 32 rows x 64 bf16
  static constexpr int SMEM_TILES = STAGES * STAGE_BYTES;
  static constexpr int SMEM_OUT = EPI_WARPS * OUT_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 2 * ACC_BUFS + 1;
  static constexpr int SMEM_BYTES = 1024 + SMEM_TILES + SMEM_OUT + NUM_BARS * 8 + 16;
  static_assert(SMEM_BYTES <= 232448, "more shared memory than one sm_100 CTA can have");
  static_assert(TMEM_COLS <= 512, "TMEM has 512 columns");
};

enum WaitSite : uint32_t {
  kWaitEmpty = 1,
  kWaitFull = 2,
  kWaitAccEmpty = 3,
  kWaitAccFull = 4,
  kWaitDrain = 5,
  kWaitMmaDone = 6,
};

struct UnitCoord {
  int tile, tm, tn, kt0, kt1, split;
};

// Unit u = split * tiles + tile; tiles are rasterised in groups of group_m
// tile rows (the reference's order, blockfp8 csrc/gemm_kernel.cuh:120-125).
__device__ __forceinline__ UnitCoord unit_coord(const GemmParams& p, int u) {
  UnitCoord c;
  c.tile = u % p.tiles;
  c.split = u / p.tiles;
  const int span = p.group_m * p.tiles_n;
  const int first_m = (c.tile / span) * p.group_m;
  const int rows = min(p.tiles_m - first_m, p.group_m);
  c.tm = first_m + (c.tile % span) % rows;
  c.tn = (c.tile % span) / rows;
  c.kt0 = c.split * p.k_per_split;
  c.kt1 = min(p.k_tiles, c.kt0 + p.k_per_split);
  return c;
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1) gemm_kernel(const __grid_constant__ GemmParams p) {
  constexpr int BN = Cfg::BN, STAGES = Cfg::STAGES, ACC_BUFS = Cfg::ACC_BUFS, COLS = Cfg::COLS;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles need 1024-byte alignment
  uint8_t* smem = smem_raw + (base - raw);
  const uint32_t s_tiles = base;
  const uint32_t s_out = base + Cfg::SMEM_TILES;
  const uint32_t s_bars = s_out + Cfg::SMEM_OUT;
  auto full = [&](int s) { return s_bars + 8u * s; };
  auto empty = [&](int s) { return s_bars + 8u * (STAGES + s); };
  auto acc_full = [&](int a) { return s_bars + 8u * (2 * STAGES + a); };
  auto acc_empty = [&](int a) { return s_bars + 8u * (2 * STAGES + ACC_BUFS + a); };
  const uint32_t mma_done = s_bars + 8u * (2 * STAGES + 2 * ACC_BUFS);
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + Cfg::SMEM_TILES + Cfg::SMEM_OUT + 8 * Cfg::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(misc + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int a = 0; a < ACC_BUFS; ++a) {
      mbar_init(acc_full(a), 1);
      mbar_init(acc_empty(a), Cfg::EPI_WARPS);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.map_a);
    tma_prefetch_desc(&p.map_b);
    tma_prefetch_desc(&p.map_c);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(misc), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = misc[0];

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = p.stream_b ? policy_evict_first() : policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
        const UnitCoord c = unit_coord(p, u);
        for (int kt = c.kt0; kt < c.kt1; ++kt) {
          if (!mbar_wait(empty(stage), phase ^ 1u, abort_flag, kWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t dst = s_tiles + uint32_t(stage) * Cfg::STAGE_BYTES;
          mbar_arrive_expect_tx(full(stage), Cfg::STAGE_BYTES);
          tma_load_2d(dst, &p.map_a, kt * 128, c.tm * 128, full(stage), pol_a);
          tma_load_2d(dst + Cfg::A_BYTES, &p.map_b, kt * 128, c.tn * BN, full(stage), pol_b);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every issued copy must land before the CTA exits (on the normal path
      // the MMA thread has already seen them all).
      const int pending = issued < STAGES ? issued : STAGES;
      for (int i = 0; i < pending; ++i) {
        if (stage == 0) {
          stage = STAGES - 1;
          phase ^= 1u;
        } else {
          --stage;
        }
        mbar_wait(full(stage), phase, nullptr, kWaitDrain);
      }
    }
    __syncwarp();  // reconverge before the CTA-wide barrier (bar.sync is .aligned)
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
        const UnitCoord c = unit_coord(p, u);
        for (int kt = c.kt0; kt < c.kt1; ++kt) {
          if (!mbar_wait(acc_empty(acc), acc_phase ^ 1u, abort_flag, kWaitAccEmpty) ||
              !mbar_wait(full(stage), phase, abort_flag, kWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = s_tiles + uint32_t(stage) * Cfg::STAGE_BYTES;
          const uint32_t b_addr = a_addr + Cfg::A_BYTES;
          const uint32_t d = tmem_base + uint32_t(acc * BN);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f8(d, smem_desc_k128_sw128(a_addr + 32 * k), smem_desc_k128_sw128(b_addr + 32 * k),
                   idesc, k > 0 ? 1u : 0u);
          mma_commit(empty(stage));   // the smem stage is free once these MMAs are done
          mma_commit(acc_full(acc));  // ... and the partial sums are in TMEM
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (++acc == ACC_BUFS) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
      }
      // All MMAs of this thread complete before TMEM is freed.
      mma_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, kWaitMmaDone);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ promotion + epilogue
    const int ew = warp - 2;     // epilogue warp 0 .. EPI_WARPS - 1
    const int g = ew >> 2;       // warpgroup: column block g * COLS .. + COLS
    const int quarter = warp & 3;  // TMEM lanes (= tile rows) 32 * quarter ..
    const int row = 32 * quarter + lane;
    const uint32_t t_lane = tmem_base + (uint32_t(32 * quarter) << 16);
    const uint32_t out_buf = s_out + uint32_t(ew) * Cfg::OUT_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;

    for (int u = blockIdx.x; u < p.units; u += gridDim.x) {
      const UnitCoord c = unit_coord(p, u);
      const int m = c.tm * 128 + row;
      const bool row_ok = m < p.M;
      const bool warp_rows = c.tm * 128 + 32 * quarter < p.M;  // warp-uniform
      const int col0 = c.tn * BN + g * COLS;
      const bool cols_ok = col0 < p.N;                         // warp-uniform
      const float* sap = p.sa + int64_t(row_ok ? m : 0) * p.sa_m;
      const float* sbp = p.sb + int64_t(cols_ok ? col0 / 128 : 0) * p.sb_n;

      float accum[COLS];
#pragma unroll
      for (int j = 0; j < COLS; ++j) accum[j] = 0.f;

      float sa_next = 0.f, sb_next = 0.f;
      if (c.kt0 < c.kt1) {
        if (row_ok) sa_next = __ldg(sap + int64_t(c.kt0) * p.sa_k);
        if (cols_ok) sb_next = __ldg(sbp + int64_t(c.kt0) * p.sb_k);
      }
      for (int kt = c.kt0; kt < c.kt1; ++kt) {
        // A K block's combined scale, as the reference forms it: sa * sb in fp32.
        const float scale = sa_next * sb_next;
        if (kt + 1 < c.kt1) {
          if (row_ok) sa_next = __ldg(sap + int64_t(kt + 1) * p.sa_k);
          if (cols_ok) sb_next = __ldg(sbp + int64_t(kt + 1) * p.sb_k);
        }
        ok = mbar_wait(acc_full(acc), acc_phase, abort_flag, kWaitAccFull) && ok;
        tc_fence_after();
        if (warp_rows && cols_ok) {
          const uint32_t t = t_lane + uint32_t(acc * BN + g * COLS);
#pragma unroll
          for (int ch = 0; ch < COLS / 32; ++ch) {
            float part[32];
            tmem_ld32(t + 32 * ch, part);
#pragma unroll
            for (int j = 0; j < 32; ++j) accum[32 * ch + j] = fmaf(part[j], scale, accum[32 * ch + j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty(acc));
        if (++acc == ACC_BUFS) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }

      bool store = warp_rows && cols_ok;
      if (p.splits > 1) {
        // Deterministic split-K: publish this split's partial, count arrivals;
        // the last CTA of the tile sums all partials in split order.
        float* ws_tile = p.workspace + int64_t(c.tile) * (128 * BN) + row * BN + g * COLS;
        const int64_t split_stride = int64_t(p.tiles) * (128 * BN);
        if (row_ok && cols_ok && ok) {
#pragma unroll
          for (int j = 0; j < COLS; j += 4)
            __stcg(reinterpret_cast<float4*>(ws_tile + c.split * split_stride + j),
                   make_float4(accum[j], accum[j + 1], accum[j + 2], accum[j + 3]));
        }
        __threadfence();
        named_bar_sync(1, Cfg::EPI_THREADS);
        if (ew == 0 && lane == 0) *last_flag = atomicAdd(p.counters + c.tile, 1) == p.splits - 1;
        named_bar_sync(1, Cfg::EPI_THREADS);
        const bool last = *last_flag != 0;
        store = store && last;
        if (last) {
          __threadfence();
          if (row_ok && cols_ok) {
#pragma unroll
            for (int j = 0; j < COLS; j += 4) {
              float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
              for (int s = 0; s < p.splits; ++s) {
                const float4 t = s == c.split
                                     ? make_float4(accum[j], accum[j + 1], accum[j + 2], accum[j + 3])
                                     : __ldcg(reinterpret_cast<const float4*>(ws_tile + s * split_stride + j));
                x.x += t.x;
                x.y += t.y;
                x.z += t.z;
                x.w += t.w;
              }
              accum[j] = x.x;
              accum[j + 1] = x.y;
              accum[j + 2] = x.z;
              accum[j + 3] = x.w;
            }
          }
          if (ew == 0 && lane == 0) p.counters[c.tile] = 0;  // ready for the next launch
        }
      }

      if (store && ok) {
        // bf16 rows -> 128B-swizzled [32 x 64] staging tile -> TMA store.
#pragma unroll
        for (int ch = 0; ch < COLS / 64; ++ch) {
          if (col0 + 64 * ch >= p.N) break;
          if (lane == 0) bulk_wait_read0();  // the previous store has read the buffer
          __syncwarp();
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            const float* a = accum + 64 * ch + 8 * v;
            __nv_bfloat162 b0 = __floats2bfloat162_rn(a[0], a[1]);
            __nv_bfloat162 b1 = __floats2bfloat162_rn(a[2], a[3]);
            __nv_bfloat162 b2 = __floats2bfloat162_rn(a[4], a[5]);
            __nv_bfloat162 b3 = __floats2bfloat162_rn(a[6], a[7]);
            uint4 w;
            w.x = *reinterpret_cast<uint32_t*>(&b0);
            w.y = *reinterpret_cast<uint32_t*>(&b1);
            w.z = *reinterpret_cast<uint32_t*>(&b2);
            w.w = *reinterpret_cast<uint32_t*>(&b3);
            const uint32_t dst = out_buf + uint32_t(lane) * 128u + uint32_t((v ^ (lane & 7)) * 16);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w.x), "r"(w.y),
                         "r"(w.z), "r"(w.w)
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&p.map_c, col0 + 64 * ch, c.tm * 128 + 32 * quarter, out_buf);
            bulk_commit();
          }
        }
      }
    }
    if (lane == 0) bulk_wait0();  // stores complete before the CTA retires
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace bfp8
