// Weight-streaming block-scaled FP8 GEMM for decode batches (M <= BN tokens,
// BN = 16, 32 or 64) on sm_100a:
//
//   C[m, n] = sum_kb sa[m, kb] * sb[n / 128, kb] * sum_{k in kb} A[m, k] * B[n, k]
//
// At decode sizes the weights are the only traffic that matters (N K bytes
// against M K of activations).  The kernel is built so that HBM streams
// weights without a gap, call after call:
//
// - Work: the weight tiles (128 rows) times their K blocks form one sequence
//   of W = tiles * k_tiles positions; CTA b of G takes positions
//   [W b / G, W (b + 1) / G), so with G = the SM count every SM streams the
//   same number of 16 KB weight tiles (+-1), whatever the layer's shape.  A
//   tile cut between CTAs is summed by the CTA holding its first part: the
//   later parts lie at the starts of their CTAs' ranges, so they are done
//   long before it reaches the tile at the end of its own range; each of
//   them stores its fp32 sums and adds one (release) to the tile's counter,
//   and the first part's CTA waits (bounded) for the count, then sums the
//   parts in K order from zero, its own from registers: deterministic, and
//   only a tile's owner ever waits, for parts that never wait.
// - Stages: a ring stage holds up to `group` consecutive K blocks of one
//   tile -- their weight tiles and their activation tiles -- requested
//   together on one barrier.  A 128-row x 128-byte TMA box reads 128 pieces
//   4 KB apart; asking for the next K blocks of the same rows at once keeps
//   each row's DRAM page open for 256-512 bytes (a TMA stream of single
//   boxes reaches about 4.1 TB/s on B200, of two or four 5.4-6.9 TB/s).
// - Two CTAs per SM: shared memory (<= 112 KB), TMEM (256 columns) and
//   registers leave room for a second CTA, so that the next call's CTAs
//   start while this call's are still finishing their tails.
// - Programmatic dependent launch: the kernel lets its dependent grid launch
//   at once and requests the weights of its first stages (and reads their
//   scales) before griddepcontrol.wait; weights are not written by the
//   previous kernel.  Activations, their scales, the workspace, the
//   counters and C are only touched after the wait.  Behind another call
//   the weight stream therefore starts while that call ends.
// - MMA: swapped operands -- the 128 MMA rows are weight rows, the N = BN
//   columns are tokens -- four tcgen05.mma.kind::f8f6f4 of 128 x BN x 32
//   per K block into one of the TMEM partial buffers.
// - QUANT: the activations arrive as bf16; each stage brings the [BN x 128]
//   bf16 tiles of its K blocks and two warps quantize them in shared memory
//   into the e4m3 operand (the quantization kernel's arithmetic: identical
//   codes and scales), so no separate quantization kernel runs.
//
// Warps: 0 TMA producer, 1 MMA issuer (and TMEM owner), 2-3 quantizers
// (QUANT), 4-7 promotion and epilogue (warp w reads TMEM lanes 32 (w % 4)).
// The promotion is the reference's (blockfp8 csrc/gemm_kernel.cuh:372-382):
// per K block, acc = fmaf(partial, sa * sb, acc), blocks in K order.
//
// Every mbarrier wait is bounded (ptx.cuh): a wait that gives up records a
// status code, the CTA drains what it has in flight, frees TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdint>
#include <type_traits>

#include "ptx.cuh"
#include "quant_math.cuh"

namespace bfp8 {

struct StreamParams {
  CUtensorMap map_w;  // weights [N, K] e4m3: [128 rows x 128 bytes] boxes, 128-byte swizzle
  CUtensorMap map_x;  // activations [M, K]: e4m3 [BN rows x 128 bytes] boxes, 128-byte swizzle;
                      // QUANT: bf16 [BN rows x 128 values] boxes, no swizzle
  const float* sa;    // activation scales (not QUANT)
  int64_t sa_m, sa_k;
  const float* sb;  // weight scales [ceil(N / 128), ceil(K / 128)]
  int64_t sb_n, sb_k;
  float eps;         // QUANT: floor of each group's amax
  __nv_bfloat16* c;  // output [M, N], row stride ldc
  int64_t ldc;
  float* workspace;  // parts of split tiles: [tiles][max_pieces][128 rows][MP tokens] fp32
  int* counters;     // one per weight tile, zero between launches
  int M, N, K;
  int tiles, k_tiles, max_pieces;
  int work;            // tiles * k_tiles positions (< 2^31)
  int work_q, work_r;  // work = work_q * grid + work_r
  int stages;          // ring depth
  int group;           // K blocks per stage (1 .. 4)
  int early;           // stages whose weights are requested before griddepcontrol.wait
  uint32_t stage_bytes;               // group * (weights + activation tiles [+ bf16 tiles])
  uint32_t x_bytes;                   // QUANT: one bf16 tile, min(M, BN) rows x 256 bytes
  uint32_t off_sa, off_sb, off_bars;  // shared-memory layout (bytes from the aligned base)
};

template <int BN_, bool QUANT_>
struct StreamCfg {
  static constexpr int BN = BN_;
  static constexpr bool QUANT = QUANT_;
  static_assert(BN == 16 || BN == 32 || BN == 64, "token tile");
  static constexpr int THREADS = 256;
  static constexpr int MIN_BLOCKS = BN <= 32 ? 2 : 1;  // a second CTA per SM (registers)
  static constexpr int ACC_BUFS = 256 / BN;            // TMEM partial buffers
  static constexpr int TMEM_COLS = 256;
  static constexpr int W_BYTES = 128 * 128;             // one weight tile: 128 rows x one K block
  static constexpr int A_BYTES = BN * 128;              // one e4m3 activation tile
  static constexpr int X_BYTES_MAX = QUANT ? BN * 256 : 0;  // one bf16 activation tile (M = BN)
  static_assert(A_BYTES % 1024 == 0 && W_BYTES % 1024 == 0, "tiles must stay 1024-byte aligned");
};

enum StreamWaitSite : uint32_t {
  kSWaitEmpty = 17,
  kSWaitFull = 18,
  kSWaitQuant = 19,
  kSWaitAccEmpty = 20,
  kSWaitAccFull = 21,
  kSWaitMmaDone = 22,
  kSWaitDrain = 23,
  kSWaitParts = 24,  // the owner of a split tile waiting for the other parts
};

// Number of CTAs whose range starts at or before position x.
__device__ __forceinline__ int stream_ctas_upto(const StreamParams& p, int64_t x) {
  const int64_t g = gridDim.x;
  const int64_t n = ((x + 1) * g + p.work - 1) / p.work;
  return n < g ? int(n) : int(g);
}

// Walks a CTA's positions group by group: a group is up to G consecutive K
// blocks of one tile and occupies one ring stage.
struct GroupWalk {
  int first, len;  // positions of the current group (relative to the CTA's start)
  int tile, kb;    // tile and K block of its first position
  int stage;
  uint32_t phase;  // parity of the stage's current use
  __device__ __forceinline__ void init(int tile0, int kb0) {
    first = 0;
    len = 0;
    tile = tile0;
    kb = kb0;
    stage = -1;
    phase = 1;
  }
  // Advance to the group after the current one; false past the range.
  __device__ __forceinline__ bool next(int L, int G, int k_tiles, int S) {
    first += len;
    kb += len;
    if (kb >= k_tiles) {
      kb -= k_tiles;
      ++tile;
    }
    if (first >= L) return false;
    len = min(min(G, L - first), k_tiles - kb);
    if (++stage == S) stage = 0;
    if (stage == 0) phase ^= 1u;
    return true;
  }
};

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, Cfg::MIN_BLOCKS) stream_kernel(const __grid_constant__ StreamParams p) {
  constexpr int BN = Cfg::BN, ACC = Cfg::ACC_BUFS;
  constexpr bool QUANT = Cfg::QUANT;

  // The next kernel in the stream may launch now; it waits for this grid's
  // completion before it reads anything this grid writes.
  griddep_launch_dependents();

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // 128-byte-swizzled tiles need 1024-byte alignment
  uint8_t* smem = smem_raw + (base - raw);
  const int S = p.stages, G = p.group;
  // Stage s: [G weight tiles][G e4m3 activation tiles][G bf16 tiles (QUANT;
  // min(M, BN) rows each, the rest of the token rows is zero in the e4m3 tile)]
  auto w_tile = [&](int s, int j) { return base + uint32_t(s) * p.stage_bytes + uint32_t(j) * Cfg::W_BYTES; };
  auto a_tile = [&](int s, int j) {
    return base + uint32_t(s) * p.stage_bytes + uint32_t(G * Cfg::W_BYTES + j * Cfg::A_BYTES);
  };
  auto x_tile = [&](int s, int j) {
    return base + uint32_t(s) * p.stage_bytes + uint32_t(G * (Cfg::W_BYTES + Cfg::A_BYTES)) + uint32_t(j) * p.x_bytes;
  };
  const uint32_t s_bars = base + p.off_bars;
  // full: a stage's weight tiles (and, without QUANT, its activation
  // tiles) have landed; xfull (QUANT): its bf16 tiles have; qready (QUANT):
  // its e4m3 operand is written; empty: its MMAs are done.
  auto full = [&](int s) { return s_bars + 8u * uint32_t(s); };
  auto empty = [&](int s) { return s_bars + 8u * uint32_t(S + s); };
  auto qready = [&](int s) { return s_bars + 8u * uint32_t(2 * S + s); };
  auto xfull = [&](int s) { return s_bars + 8u * uint32_t(3 * S + s); };
  auto acc_full = [&](int a) { return s_bars + 8u * uint32_t(4 * S + a); };
  auto acc_empty = [&](int a) { return s_bars + 8u * uint32_t(4 * S + ACC + a); };
  const uint32_t mma_done = s_bars + 8u * uint32_t(4 * S + 2 * ACC);
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + p.off_bars + 8u * uint32_t(4 * S + 2 * ACC + 1));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  // QUANT: positions whose token scales are in sa_s (monotonic; the
  // epilogue may trail the quantizers by many stage uses, so it reads this
  // count rather than a stage barrier's phase).
  volatile int* quantized = reinterpret_cast<volatile int*>(misc + 3);
  float* sb_s = reinterpret_cast<float*>(smem + p.off_sb);  // [span]: weight scale of each position
  float* sa_s = reinterpret_cast<float*>(smem + p.off_sa);  // [span][BN]: token scales of each position

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // This CTA's positions [start, start + L): W b / G = q b + r b / G with
  // W = q G + r (r b < G^2, 32-bit arithmetic).
  const int gdim = int(gridDim.x), b = int(blockIdx.x);
  const int start = p.work_q * b + (p.work_r * b) / gdim;
  const int L = p.work_q + (p.work_r * (b + 1)) / gdim - (p.work_r * b) / gdim;  // >= 1
  const int tile0 = start / p.k_tiles, kb0 = start - tile0 * p.k_tiles;
  const uint32_t x_tile_bytes = QUANT ? p.x_bytes : uint32_t(Cfg::A_BYTES);

  if (warp == 0 && lane == 0) {  // barriers (this thread also issues the first copies on them)
    const int nbars = 4 * S + 2 * ACC + 1;
    for (int i = 0; i < nbars; ++i) {
      const uint32_t count = (i >= 4 * S + ACC && i < 4 * S + 2 * ACC) ? 4u : 1u;  // acc_empty: four epilogue warps
      mbar_init(s_bars + 8u * uint32_t(i), count);
    }
    *abort_flag = 0;
    *quantized = 0;
    fence_barrier_init();
  }

  // Producer: the first stages' weights go out now, before the rest of the
  // set-up and before griddepcontrol.wait.
  GroupWalk pw;
  pw.init(tile0, kb0);
  int pre = 0;  // stages whose weights went out early
  const uint64_t pol_w = policy_evict_first();  // streamed once
  auto load_w = [&](const GroupWalk& g) {
    for (int j = 0; j < g.len; ++j)
      tma_load_2d(w_tile(g.stage, j), &p.map_w, (g.kb + j) * 128, g.tile * 128, full(g.stage), pol_w);
  };
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.map_w);
    tma_prefetch_desc(&p.map_x);
    while (pre < S && pre < p.early && pw.next(L, G, p.k_tiles, S)) {
      mbar_arrive_expect_tx(full(pw.stage), uint32_t(pw.len) * (Cfg::W_BYTES + (QUANT ? 0u : x_tile_bytes)));
      load_w(pw);
      ++pre;
    }
  }
  if (warp == 1) {
    tmem_alloc<1>(smem_u32(misc), Cfg::TMEM_COLS);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = misc[0];

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t pol_x = policy_evict_last();  // read by every CTA
      auto load_x = [&](const GroupWalk& g) {
        if constexpr (QUANT) mbar_arrive_expect_tx(xfull(g.stage), uint32_t(g.len) * x_tile_bytes);
        for (int j = 0; j < g.len; ++j)
          tma_load_2d(QUANT ? x_tile(g.stage, j) : a_tile(g.stage, j), &p.map_x, (g.kb + j) * 128, 0,
                      QUANT ? xfull(g.stage) : full(g.stage), pol_x);
      };
      griddep_wait();
      // The activations of the stages whose weights went out early.
      GroupWalk xw;
      xw.init(tile0, kb0);
      for (int k = 0; k < pre && xw.next(L, G, p.k_tiles, S); ++k) load_x(xw);
      int issued = pre;
      while (pw.next(L, G, p.k_tiles, S)) {
        if (!mbar_wait(empty(pw.stage), pw.phase ^ 1u, abort_flag, kSWaitEmpty)) break;
        mbar_arrive_expect_tx(full(pw.stage), uint32_t(pw.len) * (Cfg::W_BYTES + (QUANT ? 0u : x_tile_bytes)));
        load_x(pw);  // the small activation tiles first: the quantizers can start on them
        load_w(pw);
        ++issued;
      }
      // Every copy issued lands before the CTA may exit (after an abort the
      // MMA issuer has not consumed them all): wait for the last use of
      // each stage.
      for (int k = issued - S > 0 ? issued - S : 0; k < issued; ++k) {
        mbar_wait(full(k % S), uint32_t(k / S) & 1u, nullptr, kSWaitDrain);
        if (QUANT) mbar_wait(xfull(k % S), uint32_t(k / S) & 1u, nullptr, kSWaitDrain);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, BN);
      const uint64_t desc0 = smem_desc_k128_sw128(base);
      GroupWalk g;
      g.init(tile0, kb0);
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      while (ok && g.next(L, G, p.k_tiles, S)) {
        if (!mbar_wait(full(g.stage), g.phase, abort_flag, kSWaitFull)) break;
        if (QUANT && !mbar_wait(qready(g.stage), g.phase, abort_flag, kSWaitQuant)) break;
        for (int j = 0; j < g.len; ++j) {
          if (!mbar_wait(acc_empty(acc), acc_phase ^ 1u, abort_flag, kSWaitAccEmpty)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + uint32_t(acc * BN);
          const uint64_t a = desc0 + ((w_tile(g.stage, j) - base) >> 4);
          const uint64_t bd = desc0 + ((a_tile(g.stage, j) - base) >> 4);
#pragma unroll
          for (int k = 0; k < 4; ++k)  // K step of 32 e4m3 = 32 bytes = 2 descriptor units
            mma_f8<1>(d, a + 2 * k, bd + 2 * k, idesc, k > 0 ? 1u : 0u);
          mma_commit<1>(acc_full(acc));  // the K block's partial sums are in TMEM
          if (++acc == ACC) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
        if (ok) mma_commit<1>(empty(g.stage));  // the stage is free once these MMAs are done
      }
      mma_commit<1>(mma_done);  // every MMA issued completes before TMEM is freed
      mbar_wait(mma_done, 0, nullptr, kSWaitMmaDone);
    }
    __syncwarp();
  } else if (QUANT && warp < 4) {
    // ---------------------------------------------------------------- quantizers
    // Four half-warps; a task is one token's 128 values of one K block.
    const int qt = threadIdx.x - 64;
    const int lane16 = qt & 15, half = qt >> 4;
    const int M = p.M;
    // Token rows past M: zero codes in every stage's activation tiles and
    // zero scales, once (nothing else writes them).
    const int pad = BN - M;
    for (int idx = qt; idx < S * G * pad * 8; idx += 64) {
      const int t = idx / (pad * 8), rem = idx % (pad * 8);
      st_shared_v4(a_tile(t / G, t % G) + uint32_t(M + rem / 8) * 128u + uint32_t(rem % 8) * 16u, 0u, 0u, 0u, 0u);
    }
    for (int idx = qt; idx < L * pad; idx += 64) sa_s[(idx / pad) * BN + M + idx % pad] = 0.f;
    GroupWalk g;
    g.init(tile0, kb0);
    bool ok = true;
    while (g.next(L, G, p.k_tiles, S)) {
      ok = mbar_wait(xfull(g.stage), g.phase, abort_flag, kSWaitFull) && ok;
      const int tasks = g.len * M;
      // Steps of QB tasks per half-warp, all four half-warps in step (every
      // lane takes part in the shuffles): four independent groups at once
      // while at least 16 tasks remain (their shuffle and division chains
      // overlap), else one.
      auto step = [&](int t0, auto qb_tag) {
        constexpr int QB = decltype(qb_tag)::value;
        uint4 v[QB];
#pragma unroll
        for (int u = 0; u < QB; ++u) {
          const int task = t0 + half + 4 * u;
          const int j = task / M, t = task - j * M;
          v[u] = make_uint4(0u, 0u, 0u, 0u);  // zeros leave the amax alone
          if (ok && task < tasks && (g.kb + j) * 128 + lane16 * 8 < p.K)
            v[u] = ld_shared_v4(x_tile(g.stage, j) + uint32_t(t) * 256u + uint32_t(lane16) * 16u);
        }
#pragma unroll
        for (int u = 0; u < QB; ++u) {
          const int task = t0 + half + 4 * u;
          const int j = task / M, t = task - j * M;
          const GroupQuant gq = quantize_group(v[u], p.eps);
          if (task < tasks) {
            // 8 codes = half of 16-byte chunk lane16 / 2 of token row t, the
            // chunk XOR-swizzled with the row inside its 8-row group.
            const uint32_t chunk = uint32_t(lane16 >> 1) ^ uint32_t(t & 7);
            st_shared_v2(a_tile(g.stage, j) + uint32_t(t) * 128u + chunk * 16u + uint32_t(lane16 & 1) * 8u,
                         gq.codes.x, gq.codes.y);
            if (lane16 == 0) sa_s[(g.first + j) * BN + t] = gq.scale;
          }
        }
      };
      int t0 = 0;
      for (; t0 + 16 <= tasks; t0 += 16) step(t0, std::integral_constant<int, 4>());
      for (; t0 < tasks; t0 += 4) step(t0, std::integral_constant<int, 1>());
      fence_proxy_async_smem();  // the MMAs read the codes through the async proxy
      named_bar_sync(2, 64);
      if (qt == 0) {
        mbar_arrive(qready(g.stage));
        __threadfence_block();
        *quantized = g.first + g.len;  // the scales of these positions are in sa_s
      }
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- promotion + epilogue
    const int ew = warp - 4;  // = warp % 4: TMEM lanes 32 ew .. 32 ew + 31
    const int et = ew * 32 + lane;
    const int row = 32 * ew + lane;  // weight row inside the tile
    const uint32_t t_lane = tmem_base + (uint32_t(32 * ew) << 16);
    const int M = p.M, MP = (M + 3) & ~3;  // workspace tokens per row

    // Weight scales of every position: static data, read before the wait.
    for (int j = et; j < L; j += 128) {
      const int pos = start + j, t = pos / p.k_tiles;
      sb_s[j] = p.sb[int64_t(t) * p.sb_n + int64_t(pos - t * p.k_tiles) * p.sb_k];
    }
    griddep_wait();
    if constexpr (!QUANT) {
      for (int idx = et; idx < L * BN; idx += 128) {
        const int j = idx / BN, t = idx - j * BN;
        sa_s[idx] = t < M ? p.sa[int64_t(t) * p.sa_m + int64_t((kb0 + j) % p.k_tiles) * p.sa_k] : 0.f;
      }
    }
    named_bar_sync(1, 128);

    bool ok = true;
    float accum[BN];
#pragma unroll
    for (int q = 0; q < BN; ++q) accum[q] = 0.f;
    GroupWalk g;
    g.init(tile0, kb0);
    int acc = 0;
    uint32_t acc_phase = 0;
    while (g.next(L, G, p.k_tiles, S)) {
      for (int j = 0; j < g.len; ++j) {
        const int i = g.first + j, kb = g.kb + j;
        ok = mbar_wait(acc_full(acc), acc_phase, abort_flag, kSWaitAccFull) && ok;
        tc_fence_after();
        // QUANT: this position's token scales are written with its codes,
        // which the MMA behind acc_full waited for; the count is read only
        // now, so this is at most a short, bounded spin for it to become
        // visible (spinning earlier would take issue slots from the
        // quantizer warps on the same schedulers).
        if (QUANT && ok && j == 0) {
          const uint64_t t0 = globaltimer();
          while (*quantized < g.first + g.len) {
            if (*abort_flag || globaltimer() - t0 > kWaitTimeoutNs) {
              if (!*abort_flag)
                record_status((0x5Bull << 56) | (uint64_t(kSWaitQuant) << 32) | (uint64_t(blockIdx.x) << 8) | warp);
              *abort_flag = 1;
              ok = false;
              break;
            }
          }
          __threadfence_block();
        }
        if (ok) {
          // 16 or 32 columns (tokens) per TMEM load; the partial times
          // sa[token] * sb, added with one fmaf per value (packed in pairs).
          constexpr int CH = BN < 32 ? BN : 32;
          const float s_w = sb_s[i];
          const float4* sa4 = reinterpret_cast<const float4*>(sa_s + i * BN);
#pragma unroll
          for (int h = 0; h < BN / CH; ++h) {
            uint32_t part[CH];
            if constexpr (CH == 16) tmem_ld16_async(t_lane + uint32_t(acc * BN), part);
            else tmem_ld32_async(t_lane + uint32_t(acc * BN + CH * h), part);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < CH; q += 4) {
              const float4 s_a = sa4[(CH * h + q) / 4];
              float* a = accum + CH * h + q;
              fma2(a[0], a[1], __uint_as_float(part[q]), __uint_as_float(part[q + 1]), s_a.x * s_w, s_a.y * s_w);
              fma2(a[2], a[3], __uint_as_float(part[q + 2]), __uint_as_float(part[q + 3]), s_a.z * s_w,
                   s_a.w * s_w);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty(acc));  // the partial is in registers: buffer free
        if (++acc == ACC) {
          acc = 0;
          acc_phase ^= 1u;
        }
        if (kb != p.k_tiles - 1 && i != L - 1) continue;

        // ---- the end of this CTA's part of a tile
        const int n = g.tile * 128 + row;
        const bool row_ok = ok && n < p.N;
        const int64_t t0 = int64_t(g.tile) * p.k_tiles;
        const int first = stream_ctas_upto(p, t0) - 1;  // the CTA holding the tile's first position
        const int pieces = stream_ctas_upto(p, t0 + p.k_tiles - 1) - first;
        if (pieces == 1) {
          if (row_ok) {
#pragma unroll
            for (int q = 0; q < BN; ++q)
              if (q < M) p.c[int64_t(q) * p.ldc + n] = __float2bfloat16_rn(accum[q]);
          }
        } else if (b != first) {
          // A later part of the tile: its sums (row `row`, tokens contiguous,
          // 16-byte pieces) to the workspace, then one release add on the
          // tile's count; nothing waits here.
          float* ws = p.workspace + int64_t(g.tile) * p.max_pieces * (128 * MP) + row * MP;
          if (row_ok) {
            float4* w = reinterpret_cast<float4*>(ws + int64_t(b - first) * (128 * MP));
#pragma unroll
            for (int q = 0; q < BN; q += 4)
              if (q < M) __stcg(w + q / 4, make_float4(accum[q], accum[q + 1], accum[q + 2], accum[q + 3]));
          }
          // Every thread's stores are ordered before the add by the barrier
          // and the add's gpu-scope release.
          named_bar_sync(1, 128);
          if (et == 0) red_add_release_gpu(p.counters + g.tile, 1);
        } else {
          // The tile's first part, which this CTA reaches at the end of its
          // range (the later parts lie at the starts of theirs): wait,
          // bounded, for the other pieces - 1 parts, then sum the parts in K
          // order from zero -- its own from registers -- and store.
          float* ws = p.workspace + int64_t(g.tile) * p.max_pieces * (128 * MP) + row * MP;
          const int64_t piece_stride = 128 * MP;
          if (et == 0 && ok) {
            const uint64_t w0 = globaltimer();
            while (ld_acquire_gpu(p.counters + g.tile) < pieces - 1) {
              if (*abort_flag || globaltimer() - w0 > kWaitTimeoutNs) {
                if (!*abort_flag)
                  record_status((0x5Bull << 56) | (uint64_t(kSWaitParts) << 32) | (uint64_t(blockIdx.x) << 8) | warp);
                *abort_flag = 1;
                break;
              }
              __nanosleep(32);
            }
          }
          // (the acquire above, then the barrier: the other parts are visible to every thread)
          named_bar_sync(1, 128);
          {
            if (row_ok && !*abort_flag) {
              // the loads of up to PB parts in flight at once
              constexpr int PB = BN <= 16 ? 4 : 1;
#pragma unroll
              for (int q = 0; q < BN; ++q) accum[q] = 0.f + accum[q];  // part 0 added to zero
              for (int s0 = 1; s0 < pieces; s0 += PB) {
                float4 v[PB][BN / 4];
#pragma unroll
                for (int s = 0; s < PB; ++s) {
                  const float4* w = reinterpret_cast<const float4*>(ws + int64_t(s0 + s) * piece_stride);
#pragma unroll
                  for (int q = 0; q < BN / 4; ++q)
                    v[s][q] = (s0 + s < pieces && 4 * q < M) ? __ldcg(w + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int s = 0; s < PB; ++s) {
                  if (s0 + s < pieces) {
#pragma unroll
                    for (int q = 0; q < BN / 4; ++q) {
                      accum[4 * q] += v[s][q].x;
                      accum[4 * q + 1] += v[s][q].y;
                      accum[4 * q + 2] += v[s][q].z;
                      accum[4 * q + 3] += v[s][q].w;
                    }
                  }
                }
              }
#pragma unroll
              for (int q = 0; q < BN; ++q)
                if (q < M) p.c[int64_t(q) * p.ldc + n] = __float2bfloat16_rn(accum[q]);
            }
            // every other part has arrived: ready for the next launch
            if (et == 0 && !*abort_flag) p.counters[g.tile] = 0;
          }
        }
#pragma unroll
        for (int q = 0; q < BN; ++q) accum[q] = 0.f;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace bfp8
