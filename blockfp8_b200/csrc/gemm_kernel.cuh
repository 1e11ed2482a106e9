// Block-scaled FP8 GEMM for sm_100a (B200):
//
//   C[m, n] = sum_kb sa[m, kb] * sb[n / 128, kb] * sum_{k in kb} A[m, k] * B[n, k]
//
// One persistent, warp-specialised CTA per SM walks a static list of work
// units (an output tile and a range of 128-wide K blocks):
//
//   warps 0, 3  TMA producers (one thread each, alternate K blocks): the
//               operand tiles of each K block (128-byte swizzle, 128 bytes =
//               one K block per row) into a STAGES-deep shared-memory ring;
//               completion is counted in bytes on the stage's "full" mbarrier;
//   warps 1, 2  MMA issuers (one thread each, alternate K blocks): four
//               tcgen05.mma.kind::f8f6f4 (K = 32 each, e4m3 x e4m3 -> f32)
//               into one of ACC_BUFS tensor-memory (TMEM) partial buffers,
//               the first with the accumulator input disabled, so the buffer
//               holds exactly that block's unscaled partial sums; then
//               tcgen05.commit frees the smem stage and publishes the buffer;
//   warps 4..   promotion + epilogue (EPI_WG warpgroups; warp w reads TMEM
//               lanes 32 * (w % 4) ..): tcgen05.ld the partial, multiply by
//               the block's scale sa[m, kb] * sb[nb, kb] and add into fp32
//               registers with one fmaf per value -- the promotion of the
//               reference kernel (blockfp8 csrc/gemm_kernel.cuh:372-382), in
//               the same operation order -- and release the buffer.  Scales
//               are prefetched PF K blocks ahead.  After the unit's last K
//               block: round to bf16 into a swizzled smem tile, TMA store.
//
// Two operand orders.  Normal (prefill): the MMA's 128 rows are activation
// rows and its N = BN columns are weight rows.  Swapped (decode, SWAP): the
// 128 MMA rows are weight rows and N = BN (16..64) are tokens, so a decode
// batch of M <= 64 tokens does not waste 128-row MMAs and the promotion of
// a K block is spread over all 128 TMEM lanes (4 warps) instead of the one
// warp that may read lanes 0-31.  Every output element is the same sum of
// the same products in both orders.
//
// In-kernel quantization (FUSE, swapped order): the activations arrive as
// bf16.  At the start of each unit the epilogue warps quantize the unit's
// tokens x K range into a resident shared-memory copy of the B operand (the
// same 128-byte swizzle the TMA would write) plus per-token scales, with the
// arithmetic of the quantization kernel, and release it to the MMA issuers;
// the weight tiles stream into the stage ring meanwhile.  One kernel, no
// dependency on a previous one.
//
// Because every K block gets its own TMEM buffer, the MMAs of block k + 1
// run while block k is promoted.  With two epilogue warpgroups (BN = 256) a
// K block's MMAs go out per 128-column block, each with its own TMEM-buffer
// barriers, so a warpgroup promotes its block while the other block's MMAs
// still run.  With split-K the units of one tile cover disjoint K ranges;
// each writes its fp32 partial tile to a workspace and the last to arrive
// (an atomic counter) sums the partials in split order 0, 1, ..., S - 1 and
// stores the tile, as the reference does (blockfp8
// csrc/gemm_kernel.cuh:403-448): deterministic, no CTA waits for another.
// Stream-K plans cut the tiles' K blocks into equal per-CTA ranges instead;
// the parts of a tile meet the same way, summed in K order.
//
// CTA pairs (PAIR, prefill): a cluster of two CTAs computes a 256 x 256
// tile with cta_group::2 MMAs (M = 256) issued by the leader (rank 0).  Each
// CTA TMA-loads its own 128 A rows and 64 rows of each 128-column block of
// B (no multicast), and holds and promotes its 128 rows of the partial sums;
// stages and TMEM buffers are gated by the leader's barriers, and the
// leader's commits arrive on both CTAs' barriers.  Per SM a stage is 32 KB
// instead of 48 KB, so six stages fit.
//
// Row-parallel twins (TP): every configuration is also compiled for a group
// of GPUs that each hold a K slice of the same [M, N] product.  Instead of
// storing bf16, a tile's fp32 sum goes to the owning rank's partial buffer
// (NVLink peer memory); the arrival that completes the tile's count sums
// the ranks' partials in rank order and stores the bf16 tile into every
// rank's output (GemmParams tp_*).  No CTA waits for another rank inside the
// tile loop; one thread waits, bounded, at the end for this rank's output.
//
// Every mbarrier wait is bounded (ptx.cuh): on a timeout the kernel records a
// status code, drains its in-flight copies and MMAs, frees TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdint>

#include "ptx.cuh"
#include "quant_math.cuh"

namespace bfp8 {

constexpr int kTpMaxRanks = 8;  // ranks of a row-parallel group

struct GemmParams {
  CUtensorMap map_a;  // MMA A operand (128-row tiles): activations, or weights when swapped
  CUtensorMap map_b;  // MMA B operand (BN-row tiles): weights, or activations when swapped
  CUtensorMap map_c;  // C bf16 [M, N]
  const float* sa;
  int64_t sa_m, sa_k;
  const float* sb;
  int64_t sb_n, sb_k;
  float* workspace;  // split-K partial tiles: [splits][tiles][128 * BN] fp32
  int* counters;     // split-K arrivals, one per tile, zero between launches
  int M, N, K;
  int tiles_r, tiles_c, tiles;  // tiles over the MMA rows (128) and columns (BN)
  int k_tiles, k_per_split, splits;
  int units;    // tiles * splits (round-robin schedule)
  int sk_grid;  // > 0: stream-K schedule over this many CTAs (= gridDim.x)
  int64_t sk_work;  // stream-K: tiles * k_tiles K blocks in all
  int group_r;  // raster: groups of group_r row tiles, rows fastest inside a group
  int stream_b;  // 1: weights are read once (decode): L2 evict-first for them
  int pdl;       // 1: launched right behind our quantizer with programmatic dependent launch
  const __nv_bfloat16* x;  // in-kernel quantization: bf16 activations [M, K], row stride ldx
  int64_t ldx;
  float eps;  // in-kernel quantization: floor of each group's amax
  // Row-parallel reduction (TP configurations): every rank of a group
  // computes the same [M, N] over its own K slice.  Tile t belongs to rank
  // floor(t * world / tiles) (contiguous blocks); rank r's schedule is
  // rotated by tp_rot so it reaches its own block last.  Tile half w's
  // fp32 sum from rank r goes to slot [r][w] of the owner's tp_partials;
  // the arrival that completes the owner's count [2 + w] (usually the
  // owner's own) sums the slots in rank order, stores bf16 into every
  // rank's tp_out and adds one to every rank's counter [0].  At the end CTA
  // 0 advances its rank's counter [1] by this call's tile halves, waiting
  // first (bounded, with tp_wait) until counter [0] has caught up.
  int tp_world, tp_rank, tp_wait, tp_rot;
  float* tp_partials[kTpMaxRanks];               // [world][tile halves][128 * BN] fp32, per rank
  unsigned long long* tp_counters[kTpMaxRanks];  // [0] delivered, [1] consumed, [2 + w] arrivals
  __nv_bfloat16* tp_out[kTpMaxRanks];            // bf16 [M, N], row stride tp_ldo, per rank
  int64_t tp_ldo;
};

template <int BN_, int STAGES_, bool SWAP_, bool FUSE_ = false, bool PAIR_ = false, bool TP_ = false>
struct GemmCfg {
  static constexpr int BM = 128, BN = BN_, BK = 128, STAGES = STAGES_;
  // TP: the row-parallel twin of a configuration: a tile's sum goes into
  // the group's reduction (GemmParams tp_*) instead of a bf16 store.
  static constexpr bool TP = TP_;
  static constexpr bool SWAP = SWAP_;
  static constexpr bool FUSE = FUSE_;
  // PAIR: a cluster of two CTAs on a 256 x BN tile with cta_group::2 MMAs
  // (M = 256): each CTA loads its 128 A rows and half of each B column block,
  // holds its 128 rows of the partial sums in its TMEM and promotes them.
  static constexpr bool PAIR = PAIR_;
  static_assert(!PAIR || (!SWAP && !FUSE && BN == 256), "CTA pairs: normal order, 256-wide tiles");
  static constexpr int CG = PAIR ? 2 : 1;          // tcgen05 CTA group
  static constexpr int TILE_M = PAIR ? 256 : 128;  // MMA rows of a tile
  static_assert(SWAP ? (BN == 16 || BN == 32 || BN == 64) : (BN == 64 || BN == 128 || BN == 256),
                "unsupported tile");
  static_assert(!FUSE || SWAP, "in-kernel quantization needs the swapped order");
  static constexpr int COLS = SWAP ? BN : (BN < 128 ? BN : 128);  // accumulators per thread
  static constexpr int EPI_WG = SWAP ? 1 : BN / COLS;
  static constexpr int EPI_WARPS = 4 * EPI_WG;
  static constexpr int EPI_THREADS = 32 * EPI_WARPS;
  // Warpgroup 0: TMA producers (warps 0, 3) and MMA issuers (warps 1, 2);
  // warpgroups 1.. the epilogue, so registers can move between the roles by
  // warpgroup.
  static constexpr int THREADS = 128 + EPI_THREADS;
  // Register split (setmaxnreg) when the launch share is too small for the
  // epilogue's 128 accumulators: warpgroup 0 gives up all but REG_LOW.
  static constexpr int REGS_LAUNCH = (65536 / THREADS) / 8 * 8 > 255 ? 255 : (65536 / THREADS) / 8 * 8;
  // 64 for warpgroup 0: its scheduling loops spill below that (measured:
  // the 256 x 256 pair configuration runs 5% faster than with 40); the
  // epilogue's 128 accumulators and two 32-column TMEM chunks fit in 216.
  static constexpr int REG_LOW = 64;
  static constexpr int REG_HIGH_FIT = ((REGS_LAUNCH * THREADS - 128 * REG_LOW) / EPI_THREADS) / 8 * 8;
  static constexpr int REG_HIGH = REG_HIGH_FIT > 216 ? 216 : REG_HIGH_FIT;
  static constexpr bool SPLIT_REGS = REGS_LAUNCH < 200;
  static_assert(!SPLIT_REGS || 128 * REG_LOW + EPI_THREADS * REG_HIGH <= REGS_LAUNCH * THREADS,
                "register split exceeds the launch allocation");
  // TMEM partial buffers: as many as fit (up to 16), so for small tiles the
  // MMAs can run far ahead of a unit's epilogue (split-K hand-off, store).
  static constexpr int ACC_BUFS = 512 / BN > 16 ? 16 : 512 / BN;
  static constexpr int TMEM_COLS = ACC_BUFS * BN < 32 ? 32 : ACC_BUFS * BN;
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK;  // this CTA's rows of the B tile
  // FUSE: the B operand of a whole unit stays resident (ACT_KB K blocks at
  // most, 64 KB), so the ring only carries weight tiles.
  static constexpr int ACT_KB = FUSE ? 65536 / B_BYTES : 0;
  static constexpr int SMEM_ACT = ACT_KB * B_BYTES;
  static constexpr int SMEM_ACT_SCALES = ACT_KB * BN * 4;
  static constexpr int STAGE_BYTES = FUSE ? A_BYTES : A_BYTES + B_BYTES;
  // Output staging per epilogue warp: normal, two [32 rows x 32 bf16] chunk
  // buffers (64-byte swizzle); swapped, one [BN tokens x 32 bf16] tile.
  static constexpr int OUT_BYTES = SWAP ? BN * 64 : 2 * 32 * 64;
  static constexpr int SMEM_TILES = STAGES * STAGE_BYTES;
  static constexpr int SMEM_OUT = ((EPI_WARPS * OUT_BYTES + 1023) / 1024) * 1024;
  // Each epilogue warpgroup owns a column block of the tile and its own pair
  // of TMEM-buffer barriers; the MMAs of a K block go out per column block,
  // so a warpgroup can promote its block while the next block's MMAs run.
  static constexpr int COL_BLOCKS = EPI_WG;
  static constexpr int BN_CB = BN / COL_BLOCKS;                  // MMA N of a column block
  static constexpr int B_ROWS_CB = PAIR ? BN_CB / 2 : BN_CB;     // its B rows in this CTA
  static constexpr int NUM_BARS = 2 * STAGES + 2 * ACC_BUFS * COL_BLOCKS + 1 + ACT_KB;
  static constexpr int ACT_RING = ACT_KB > 0 ? ACT_KB : 1;  // act_ready barriers (FUSE), at least 1 for the modulo
  static constexpr int SMEM_MISC = 16 + 4 * STAGES;  // TMEM slot, flags, last load per stage
  static constexpr int SMEM_BYTES =
      1024 + SMEM_TILES + SMEM_ACT + SMEM_OUT + SMEM_ACT_SCALES + NUM_BARS * 8 + SMEM_MISC;
  static_assert(SMEM_BYTES <= 232448, "more shared memory than one sm_100 CTA can have");
  // Two producers and two MMA issuers take alternate K blocks.  With an even
  // number of stages and of TMEM buffers, each stage and each buffer always
  // belongs to the same producer and the same issuer, so a thread's wait on a
  // barrier is never two phases ahead of it (a parity wait would then pass on
  // the stale phase).  With an odd count, an issuer could reach stage s's
  // next round while the other producer had not yet refilled it.
  static_assert(STAGES % 2 == 0 && ACC_BUFS % 2 == 0, "stages and TMEM buffers must come in pairs");
  static_assert(TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation");
  static_assert(STAGE_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "tiles must stay 1024-byte aligned");
};

// The row-parallel twin of configuration C.
template <class C>
using WithTp = GemmCfg<C::BN, C::STAGES, C::SWAP, C::FUSE, C::PAIR, true>;

enum WaitSite : uint32_t {
  kWaitEmpty = 1,
  kWaitFull = 2,
  kWaitAccEmpty = 3,
  kWaitAccFull = 4,
  kWaitDrain = 5,
  kWaitMmaDone = 6,
  kWaitActReady = 7,  // a resident activation K block (FUSE)
  kWaitTpDelivered = 8,  // row-parallel: the other ranks' tiles of this rank's output
};

// A unit: one tile's K blocks kt0 .. kt1 - 1, the part `split` of the tile's
// `pieces` parts (pieces > 1: partial sums meet in the workspace).
struct UnitCoord {
  int tile, tr, tc, kt0, kt1, split, pieces;
  int stile;  // the tile's place in the schedule (= tile unless a row-parallel rank rotates it)
};

// Two schedules of a CTA's units.
// Round-robin split-K: unit u = split * tiles + tile, CTA b takes
// u = b, b + gridDim.x, ... below p.units.
// Stream-K (p.sk_grid > 0): the tiles' K blocks in one sequence (position
// tile * k_tiles + kt), CTA b takes positions [W b / G, W (b + 1) / G) with
// W = p.sk_work and G = p.sk_grid, so every CTA streams the same number of
// K blocks (+-1); a unit is the part of one tile inside that range and u
// is its first position.  The parts of a tile are numbered in K order.
__device__ __forceinline__ int64_t sk_begin(const GemmParams& p, int b) {
  return int64_t(b) * p.sk_work / p.sk_grid;
}
// Number of CTAs whose range starts at or before position x.
__device__ __forceinline__ int sk_starts_upto(const GemmParams& p, int64_t x) {
  const int64_t n = ((x + 1) * p.sk_grid + p.sk_work - 1) / p.sk_work;
  return n < p.sk_grid ? int(n) : p.sk_grid;
}
// sid / scount: this CTA's (or CTA pair's) index among scount schedulers.
__device__ __forceinline__ int first_unit(const GemmParams& p, int sid) {
  return p.sk_grid > 0 ? int(sk_begin(p, sid)) : sid;
}
__device__ __forceinline__ bool unit_valid(const GemmParams& p, int u, int sid) {
  return p.sk_grid > 0 ? u < sk_begin(p, sid + 1) : u < p.units;
}

// Tiles are rasterised in groups of group_r row tiles, row tiles fastest
// inside a group (the reference's order, blockfp8
// csrc/gemm_kernel.cuh:120-125); the host picks group_r so the operand that
// is re-read stays in L2.
__device__ __forceinline__ UnitCoord unit_coord(const GemmParams& p, int u, int sid) {
  UnitCoord c;
  if (p.sk_grid > 0) {
    c.tile = u / p.k_tiles;
    c.kt0 = u % p.k_tiles;
    const int64_t end = c.kt0 + (sk_begin(p, sid + 1) - u);
    c.kt1 = end < p.k_tiles ? int(end) : p.k_tiles;
    const int64_t t0 = int64_t(c.tile) * p.k_tiles;
    const int before = sk_starts_upto(p, t0);
    c.split = sk_starts_upto(p, u) - before;
    c.pieces = sk_starts_upto(p, t0 + p.k_tiles - 1) - before + 1;
  } else {
    c.tile = u % p.tiles;
    c.split = u / p.tiles;
    c.kt0 = c.split * p.k_per_split;
    c.kt1 = min(p.k_tiles, c.kt0 + p.k_per_split);
    c.pieces = p.splits;
  }
  c.stile = c.tile;
  if (p.tp_rot) c.tile = (c.tile + p.tp_rot) % p.tiles;
  const int span = p.group_r * p.tiles_c;
  const int first = (c.tile / span) * p.group_r;
  const int rows = min(p.tiles_r - first, p.group_r);
  c.tr = first + (c.tile % span) % rows;
  c.tc = (c.tile % span) / rows;
  return c;
}

__device__ __forceinline__ int next_unit(const GemmParams& p, int u, const UnitCoord& c, int scount) {
  return p.sk_grid > 0 ? c.stile * p.k_tiles + c.kt1 : u + scount;
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[N]);
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, float (&v)[32]) {
  tmem_ld32(taddr, v);
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float (&v)[16]) {
  tmem_ld16(taddr, v);
}

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// In-kernel quantization of one unit's activations (FUSE): the tokens
// tok0 .. tok0 + BN - 1 over K blocks kt0 .. kt1 - 1 become the unit's
// resident B operand (one [BN x 128 B] 128-byte-swizzled tile per K block
// at s_act + k * B_BYTES) and scales (s_act_scales[k * BN + token]).  Token
// rows past M get zero codes and a zero scale with no load and no division.
// The real (K block, token) groups go in K-block order to half-warps, QB
// groups per half-warp per batch, the next batch's loads in flight while
// this one is converted; after each batch the K blocks it completed are
// released to the MMA issuers one by one, so the first MMAs start after the
// first batch.  The K block at position q of the CTA's K-block sequence
// (seq_base + k for the unit's block k) is released on act_ready[q % ACT_KB],
// whose phase (q / ACT_KB) it completes: every position is released once, a
// barrier serves positions ACT_KB apart -- the same MMA issuer (ACT_KB is
// even), never two of one unit (no unit is longer) -- so an issuer's parity
// wait is never a phase ahead of or behind the barrier.  Real tokens get the
// quantization kernel's arithmetic: amax from eps, IEEE amax / 448, clamp,
// round-to-nearest-even e4m3 with saturation.
template <class Cfg>
__device__ __forceinline__ void quantize_unit(const GemmParams& p, const UnitCoord& c, uint32_t s_act,
                                              uint32_t s_act_scales, uint32_t act_ready0, int seq_base,
                                              int ethread) {
  constexpr int BN = Cfg::BN, QB = 8;
  constexpr int ET = Cfg::EPI_THREADS, HALVES = ET / 16, STEP = HALVES * QB;
  const int lane16 = ethread & 15, half = ethread >> 4;
  const int tok0 = c.tc * BN;
  const int rows = min(BN, p.M - tok0);
  const int nkb = c.kt1 - c.kt0;
  const int groups = nkb * rows;

  // Padding token rows: zero codes (16 bytes per thread per step) and scales.
  const int pad_units = nkb * (BN - rows) * 8;  // 16-byte units
  for (int i = ethread; i < pad_units; i += ET) {
    const int kl = i / ((BN - rows) * 8), rem = i % ((BN - rows) * 8);
    const int row = rows + rem / 8, unit = rem % 8;
    st_shared_v4(s_act + uint32_t(kl) * Cfg::B_BYTES + uint32_t(row) * 128u + uint32_t(unit) * 16u, 0u, 0u,
                 0u, 0u);
  }
  for (int i = ethread; i < nkb * (BN - rows); i += ET) {
    const int kl = i / (BN - rows), row = rows + i % (BN - rows);
    st_shared_f32(s_act_scales + uint32_t(kl * BN + row) * 4u, 0.f);
  }

  auto load = [&](uint4 (&v)[QB], int g0) {
#pragma unroll
    for (int b = 0; b < QB; ++b) {
      const int gi = g0 + half + b * HALVES;
      const int kl = gi / rows, row = gi % rows;
      const int col = (c.kt0 + kl) * 128 + lane16 * 8;
      v[b] = make_uint4(0u, 0u, 0u, 0u);  // past K: zeros, which leave the amax alone
      if (gi < groups && col < p.K)
        v[b] = __ldg(reinterpret_cast<const uint4*>(p.x + int64_t(tok0 + row) * p.ldx + col));
    }
  };
  uint4 cur[QB], nxt[QB];
  load(cur, 0);
  int released = 0;  // K blocks of this unit already handed to the MMA issuers
  // Every thread walks the same batches (the shuffle needs all 32 lanes).
  for (int g0 = 0; g0 < groups; g0 += STEP) {
    if (g0 + STEP < groups) load(nxt, g0 + STEP);
#pragma unroll
    for (int b = 0; b < QB; ++b) {
      const int gi = g0 + half + b * HALVES;
      const int kl = gi / rows, row = gi % rows;
      const GroupQuant gq = quantize_group(cur[b], p.eps);  // all 32 lanes (shuffles)
      if (gi < groups) {
        const float scale = gq.scale;
        const uint32_t packed[2] = {gq.codes.x, gq.codes.y};
        // 8 codes of chunk lane16 of token row `row`: 16-byte unit lane16 / 2
        // of the row, XOR-swizzled with the row inside its 8-row group.
        const uint32_t unit16 = uint32_t(lane16 >> 1) ^ uint32_t(row & 7);
        st_shared_v2(s_act + uint32_t(kl) * Cfg::B_BYTES + uint32_t(row) * 128u + unit16 * 16u +
                         uint32_t(lane16 & 1) * 8u,
                     packed[0], packed[1]);
        if (lane16 == 0) st_shared_f32(s_act_scales + uint32_t(kl * BN + row) * 4u, scale);
      }
    }
    fence_proxy_async_smem();  // the MMAs read the operand through the async proxy
    named_bar_sync(1, ET);
    const int done = min(nkb, min(groups, g0 + STEP) / rows);  // whole K blocks finished
    if (ethread == 0)
      for (; released < done; ++released)
        mbar_arrive(act_ready0 + 8u * uint32_t((seq_base + released) % Cfg::ACT_RING));
    released = done;
#pragma unroll
    for (int b = 0; b < QB; ++b) cur[b] = nxt[b];
  }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1) gemm_kernel(const __grid_constant__ GemmParams p) {
  constexpr int BN = Cfg::BN, STAGES = Cfg::STAGES, ACC_BUFS = Cfg::ACC_BUFS, COLS = Cfg::COLS;
  constexpr bool SWAP = Cfg::SWAP, FUSE = Cfg::FUSE, PAIR = Cfg::PAIR;
  constexpr int CG = Cfg::CG;
  constexpr int PF = 4;  // scale prefetch distance in K blocks

  // The next kernel of the stream may launch now (programmatic dependent
  // launch); it waits for this grid's completion before it uses our output.
  griddep_launch_dependents();

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles need 1024-byte alignment
  uint8_t* smem = smem_raw + (base - raw);
  const uint32_t s_tiles = base;
  const uint32_t s_act = s_tiles + Cfg::SMEM_TILES;  // FUSE: the unit's B operand
  const uint32_t s_out = s_act + Cfg::SMEM_ACT;
  const uint32_t s_act_scales = s_out + Cfg::SMEM_OUT;  // FUSE: [ACT_KB][BN] fp32
  const uint32_t s_bars = s_act_scales + Cfg::SMEM_ACT_SCALES;
  auto full = [&](int s) { return s_bars + 8u * s; };
  auto empty = [&](int s) { return s_bars + 8u * (STAGES + s); };
  constexpr int CB = Cfg::COL_BLOCKS;
  auto acc_full = [&](int a, int h) { return s_bars + 8u * (2 * STAGES + a * CB + h); };
  auto acc_empty = [&](int a, int h) { return s_bars + 8u * (2 * STAGES + (ACC_BUFS + a) * CB + h); };
  const uint32_t mma_done = s_bars + 8u * (2 * STAGES + 2 * ACC_BUFS * CB);
  const uint32_t act_ready0 = mma_done + 8u;  // FUSE: [ACT_KB], by position
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + (s_bars - base) + 8 * Cfg::NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(misc + 2);
  volatile int* stage_seq = reinterpret_cast<volatile int*>(misc + 4);  // last K block loaded per stage

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Scheduling: a CTA pair walks the units together (cluster rank 0 leads:
  // its barriers gate the stages and TMEM buffers, its thread issues the MMAs).
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  const int sid = PAIR ? int(blockIdx.x >> 1) : int(blockIdx.x);
  const int scount = PAIR ? int(gridDim.x >> 1) : int(gridDim.x);
  const int row_off = PAIR ? int(rank) * 128 : 0;  // this CTA's first row inside a tile
  // The leader's copy of one of this CTA's barriers (same offset).
  auto leader_bar = [&](uint32_t bar) { return PAIR ? map_shared_rank(bar, 0) : bar; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int a = 0; a < ACC_BUFS; ++a)
      for (int h = 0; h < CB; ++h) {
        mbar_init(acc_full(a, h), 1);
        // the four warps of column block h's warpgroup (of both CTAs of a pair)
        mbar_init(acc_empty(a, h), PAIR ? 8 : 4);
      }
    mbar_init(mma_done, 2);  // one commit from each MMA issuer
    for (int k = 0; k < Cfg::ACT_KB; ++k) mbar_init(act_ready0 + 8u * k, 1);  // FUSE: activations in place
    *abort_flag = 0;
    for (int st = 0; st < STAGES; ++st) stage_seq[st] = -1;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.map_a);
    if constexpr (!FUSE) tma_prefetch_desc(&p.map_b);
    tma_prefetch_desc(&p.map_c);
  }
  if (warp == 1) {
    tmem_alloc<CG>(smem_u32(misc), Cfg::TMEM_COLS);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();  // the peer's barriers are initialised before any remote use
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = misc[0];

  if (warp < 4) {
    if constexpr (Cfg::SPLIT_REGS) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Cfg::REG_LOW));
    // Two TMA producers (warps 0 and 3) and two MMA issuers (warps 1 and 2),
    // one thread each, take alternate K blocks of the CTA's sequence: the
    // per-K-block cost of the barrier tests and instruction issue is paid by
    // two threads in parallel.  K block i of the sequence always uses smem
    // stage i % STAGES (phase (i / STAGES) & 1) and TMEM buffer i % ACC_BUFS
    // (phase (i / ACC_BUFS) & 1), whoever handles it.
    const bool producer = warp == 0 || warp == 3;
    const int role = (warp == 0 || warp == 1) ? 0 : 1;  // which half of the K blocks
    if (lane == 0) {
      if (producer) {
        // ------------------------------------------------------------ TMA producer
        // Activations are re-read by many tiles: keep them; weights streamed
        // once (decode) go first.
        const uint64_t pol_act = policy_evict_last();
        const uint64_t pol_wgt = p.stream_b ? policy_evict_first() : policy_evict_normal();
        // Weights are operand A when swapped, B otherwise.  After our own
        // quantizer (p.pdl, programmatic dependent launch) the weight tiles
        // of this thread's first K blocks (among the first STAGES) go out
        // before griddepcontrol.wait, so they stream while the quantizer
        // finishes; activation tiles only after it.  FUSE: the ring carries
        // weight tiles only.
        const CUtensorMap* map_w = SWAP ? &p.map_a : &p.map_b;
        const CUtensorMap* map_x = SWAP ? &p.map_b : &p.map_a;
        const uint32_t off_w = SWAP ? 0u : uint32_t(Cfg::A_BYTES);
        const uint32_t off_x = SWAP ? uint32_t(Cfg::A_BYTES) : 0u;
        // A pair's stage completes on the leader's barrier with both CTAs' bytes.
        constexpr uint32_t kFullBytes = Cfg::STAGE_BYTES * (PAIR ? 2 : 1);
        auto w_row = [&](const UnitCoord& c) { return SWAP ? c.tr * 128 : c.tc * BN; };
        auto x_row = [&](const UnitCoord& c) { return SWAP ? c.tc * BN : c.tr * Cfg::TILE_M + row_off; };
        // Weight tile of a K block: the BN rows, or for a pair this CTA's
        // B_ROWS_CB-row share of each column block (rows h * BN_CB + rank * B_ROWS_CB).
        auto load_w = [&](uint32_t dst, int kt, const UnitCoord& c, int stage, uint64_t pol) {
          if constexpr (PAIR) {
#pragma unroll
            for (int h = 0; h < CB; ++h)
              tma_load_2d_pair(dst + off_w + uint32_t(h * Cfg::B_ROWS_CB * 128), map_w, kt * 128,
                               w_row(c) + h * Cfg::BN_CB + int(rank) * Cfg::B_ROWS_CB, leader_bar(full(stage)),
                               pol);
          } else {
            tma_load_2d(dst + off_w, map_w, kt * 128, w_row(c), full(stage), pol);
          }
        };
        auto load_x = [&](uint32_t dst, int kt, const UnitCoord& c, int stage, uint64_t pol) {
          if constexpr (PAIR) tma_load_2d_pair(dst + off_x, map_x, kt * 128, x_row(c), leader_bar(full(stage)), pol);
          else tma_load_2d(dst + off_x, map_x, kt * 128, x_row(c), full(stage), pol);
        };
        int early = 0;  // K blocks (of the whole sequence) whose weights went out early
        if (p.pdl && !FUSE) {
          int seq = 0;
          for (int u = first_unit(p, sid); unit_valid(p, u, sid) && seq < STAGES;) {
            const UnitCoord c = unit_coord(p, u, sid);
            u = next_unit(p, u, c, scount);
            for (int kt = c.kt0; kt < c.kt1 && seq < STAGES; ++kt, ++seq) {
              if ((seq & 1) != role) continue;
              const uint32_t dst = s_tiles + uint32_t(seq) * Cfg::STAGE_BYTES;  // stage = seq
              if (leader) mbar_arrive_expect_tx(full(seq), kFullBytes);
              load_w(dst, kt, c, seq, pol_wgt);
              stage_seq[seq] = seq;
            }
          }
          early = seq;
        }
        if (!FUSE) griddep_wait();  // activations are the previous kernel's output
        int seq = 0;
        bool ok = true;
        for (int u = first_unit(p, sid); ok && unit_valid(p, u, sid);) {
          const UnitCoord c = unit_coord(p, u, sid);
          u = next_unit(p, u, c, scount);
          for (int kt = c.kt0; kt < c.kt1; ++kt, ++seq) {
            if ((seq & 1) != role) continue;
            const int stage = seq % STAGES;
            const uint32_t dst = s_tiles + uint32_t(stage) * Cfg::STAGE_BYTES;
            if (seq < early) {  // weights already requested; add the activations
              load_x(dst, kt, c, stage, pol_act);
              continue;
            }
            const uint32_t phase = uint32_t(seq / STAGES) & 1u;
            if (!mbar_wait(empty(stage), phase ^ 1u, abort_flag, kWaitEmpty)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(full(stage), kFullBytes);
            load_w(dst, kt, c, stage, pol_wgt);
            if constexpr (!FUSE) load_x(dst, kt, c, stage, pol_act);
            stage_seq[stage] = seq;
          }
        }
      } else if (leader) {
        // ------------------------------------------------------------ MMA issuer
        // (a pair's MMAs are issued by the leader for both CTAs)
        constexpr int BN_CB = Cfg::BN_CB;
        constexpr uint32_t idesc = idesc_e4m3_f32(Cfg::TILE_M, BN_CB);
        // Commits arrive on this CTA's barrier and, for a pair, on the peer's.
        auto commit_both = [&](uint32_t bar) {
          mma_commit<CG>(bar);
          if constexpr (PAIR) mma_commit<CG>(map_shared_rank(bar, 1));
        };
        // Descriptors of stage 0's tiles; a stage, a resident K block or a K
        // step only moves the 14-bit start-address field (16-byte units),
        // which never carries out (shared memory ends below 256 KB).
        const uint64_t desc_a0 = smem_desc_k128_sw128(s_tiles);
        const uint64_t desc_b0 = smem_desc_k128_sw128(FUSE ? s_act : s_tiles + Cfg::A_BYTES);
        int seq = 0;
        bool ok = true;
        for (int u = first_unit(p, sid); ok && unit_valid(p, u, sid);) {
          const UnitCoord c = unit_coord(p, u, sid);
          u = next_unit(p, u, c, scount);
          for (int kt = c.kt0; kt < c.kt1; ++kt, ++seq) {
            if ((seq & 1) != role) continue;
            if (FUSE && !mbar_wait(act_ready0 + 8u * uint32_t(seq % Cfg::ACT_RING),
                                   uint32_t(seq / Cfg::ACT_RING) & 1u, abort_flag, kWaitActReady)) {
              ok = false;
              break;
            }
            const int stage = seq % STAGES, acc = seq % ACC_BUFS;
            const uint32_t phase = uint32_t(seq / STAGES) & 1u;
            const uint32_t acc_phase = uint32_t(seq / ACC_BUFS) & 1u;
            if (!mbar_wait(full(stage), phase, abort_flag, kWaitFull)) {
              ok = false;
              break;
            }
            const uint64_t a_off = uint64_t(stage) * (Cfg::STAGE_BYTES >> 4);
            const uint64_t b_off = FUSE ? uint64_t(kt - c.kt0) * (Cfg::B_BYTES >> 4) : a_off;
#pragma unroll
            for (int h = 0; h < CB; ++h) {
              if (!mbar_wait(acc_empty(acc, h), acc_phase ^ 1u, abort_flag, kWaitAccEmpty)) {
                ok = false;
                break;
              }
              tc_fence_after();
              // Column block h: TMEM columns acc * BN + h * BN_CB; its B rows
              // start B_ROWS_CB * h rows into the stage's B tile (128 bytes a row).
              const uint32_t d = tmem_base + uint32_t(acc * BN + h * BN_CB);
              const uint64_t bh = uint64_t(h) * ((Cfg::B_ROWS_CB * 128) >> 4);
#pragma unroll
              for (int k = 0; k < 4; ++k)  // K step of 32 e4m3 = 32 bytes = 2 descriptor units
                mma_f8<CG>(d, desc_a0 + a_off + 2 * k, desc_b0 + b_off + bh + 2 * k, idesc, k > 0 ? 1u : 0u);
              commit_both(acc_full(acc, h));  // column block h's partial sums are in TMEM
            }
            if (!ok) break;
            commit_both(empty(stage));  // the smem stage is free once these MMAs are done
          }
        }
        // All MMAs of both issuers complete before TMEM is freed.
        mma_commit<CG>(mma_done);
        mbar_wait(mma_done, 0, nullptr, kWaitMmaDone);
      }
    }
    __syncwarp();  // reconverge before the barriers below (bar.sync is .aligned)
    if (producer) {
      // Every issued copy must land before the CTA exits.  On the normal path
      // the MMA threads have seen them all; after an abort, wait on the last
      // load of each stage (its phase completes when its bytes arrive).
      named_bar_sync(2, 64);  // both producers are done issuing
      // (a pair's stages complete on the leader's barriers, with both CTAs' bytes)
      if (warp == 0 && lane == 0 && leader)
        for (int st = 0; st < STAGES; ++st)
          if (stage_seq[st] >= 0)
            mbar_wait(full(st), uint32_t(stage_seq[st] / STAGES) & 1u, nullptr, kWaitDrain);
      __syncwarp();
    }
  } else {
    if constexpr (Cfg::SPLIT_REGS) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(Cfg::REG_HIGH));
    // ------------------------------------------------------------ promotion + epilogue
    const int ew = warp - 4;        // epilogue warp 0 .. EPI_WARPS - 1
    const int g = ew >> 2;          // warpgroup: column block g * COLS .. + COLS
    const int quarter = warp & 3;   // TMEM lanes (= tile rows) 32 * quarter ..
    const int row = 32 * quarter + lane;
    const uint32_t t_lane = tmem_base + (uint32_t(32 * quarter) << 16);
    const uint32_t out_buf = s_out + uint32_t(ew) * Cfg::OUT_BYTES;
    const int rows_total = SWAP ? p.N : p.M;  // extent of the MMA row dimension
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    int out_chunk = 0;  // normal mode: alternates between the two staging buffers

    // Scale sources of a unit.  Normal: sa per row (thread), sb per
    // 128-column block (warpgroup g promotes column block g).  Swapped: sb per
    // 128-row tile (CTA), sa per token column; lane j loads token col0 + j
    // (and col0 + 32 + j when BN = 64).  FUSE: sa comes from the unit's
    // resident scales.
    struct ScaleSrc {
      const float* sa;
      const float* sa2;
      const float* sb;
      bool sa_ok, sa2_ok, sb_ok;
    };
    auto scale_src = [&](const UnitCoord& c) {
      ScaleSrc q{p.sa, p.sa, p.sb, false, false, false};
      const int col0 = c.tc * BN + g * COLS;
      if constexpr (!SWAP) {
        const int r = c.tr * Cfg::TILE_M + row_off + row;
        q.sa_ok = r < rows_total;
        q.sa = p.sa + int64_t(q.sa_ok ? r : 0) * p.sa_m;
        q.sb_ok = col0 < p.N;
        q.sb = p.sb + int64_t(q.sb_ok ? col0 / 128 : 0) * p.sb_n;
      } else {
        const int t0 = col0 + lane, t1 = col0 + 32 + lane;
        q.sa_ok = !FUSE && t0 < p.M && lane < BN;
        q.sa = p.sa + int64_t(q.sa_ok ? t0 : 0) * p.sa_m;
        if constexpr (BN > 32) {
          q.sa2_ok = !FUSE && t1 < p.M;
          q.sa2 = p.sa + int64_t(q.sa2_ok ? t1 : 0) * p.sa_m;
        }
        q.sb_ok = true;  // the tile's weight block exists (tr * 128 < N)
        q.sb = p.sb + int64_t(c.tr) * p.sb_n;
      }
      return q;
    };
    // Scales of a unit's K blocks kt0 + j, j < PF, ride in pa/pa2/pb[j] and
    // are refilled PF K blocks ahead of their use; the next unit's first PF
    // scales go out into na/na2/nb when the current unit starts, so they are
    // in place at the unit boundary (a load issued while the weights stream
    // at full speed can take microseconds).
    float pa[PF], pa2[PF], pb[PF], na[PF], na2[PF], nb[PF];
    auto load_scales = [&](const ScaleSrc& q, int kt, float& a, float& a2, float& b) {
      a = q.sa_ok ? ldg_pinned(q.sa + int64_t(kt) * p.sa_k) : 0.f;
      if constexpr (SWAP && BN > 32) a2 = q.sa2_ok ? ldg_pinned(q.sa2 + int64_t(kt) * p.sa_k) : 0.f;
      b = q.sb_ok ? ldg_pinned(q.sb + int64_t(kt) * p.sb_k) : 0.f;
    };
    auto prefetch_unit = [&](const UnitCoord& c, float (&a)[PF], float (&a2)[PF], float (&b)[PF]) {
      const ScaleSrc q = scale_src(c);
#pragma unroll
      for (int j = 0; j < PF; ++j)
        if (c.kt0 + j < c.kt1) load_scales(q, c.kt0 + j, a[j], a2[j], b[j]);
    };
    // FUSE: quantize a unit's activations, handing each K block to the MMA
    // issuers as soon as it is in place; seq_base = the unit's first position
    // in the CTA's K-block sequence.
    auto publish_unit = [&](const UnitCoord& c, int seq_base) {
      if constexpr (FUSE) quantize_unit<Cfg>(p, c, s_act, s_act_scales, act_ready0, seq_base, ew * 32 + lane);
    };

    if (!FUSE) griddep_wait();  // activation scales are the previous kernel's output
    const int u0 = first_unit(p, sid);
    const bool any_unit = unit_valid(p, u0, sid);
    UnitCoord c_next = unit_coord(p, any_unit ? u0 : 0, sid);
    if (any_unit) {
      prefetch_unit(c_next, pa, pa2, pb);
      publish_unit(c_next, 0);
    }

    // Row-parallel hand-off of the tiles this CTA holds whole (every
    // epilogue thread runs these; the barriers inside are CTA-wide).  A
    // partial goes in [column][row] order so a warp's stores and loads cover
    // 128 contiguous bytes, local or across NVLink.  No CTA waits here for
    // another rank: the arrival that completes a tile's count does the sum.
    auto tp_owner = [&](const UnitCoord& c) { return int(int64_t(c.tile) * p.tp_world / p.tiles); };
    auto tp_wtile = [&](const UnitCoord& c) { return PAIR ? c.tile * 2 + int(rank) : c.tile; };
    const int64_t tp_rank_stride = int64_t(p.tiles) * (PAIR ? 2 : 1) * (128 * BN);
    // Column j of a thread's accumulators is tile column tp_col(j).
    auto tp_col = [&](int j) { return SWAP ? j : g * COLS + j; };
    auto tp_slots = [&](const UnitCoord& c) {
      return p.tp_partials[tp_owner(c)] + int64_t(tp_wtile(c)) * (128 * BN) + row;
    };
    // This rank's fp32 sum of tile c into its slot at the owner.
    auto tp_push = [&](const UnitCoord& c, bool row_ok, bool cols_ok, float (&accum)[COLS], bool ok) {
      if (row_ok && cols_ok && ok) {
        float* w = tp_slots(c) + p.tp_rank * tp_rank_stride;
#pragma unroll
        for (int j = 0; j < COLS; ++j) __stcg(w + tp_col(j) * 128, accum[j]);
      }
    };
    // One arrival on tile c (after every thread's push, by the barrier);
    // true, on every thread, for the arrival that completes the count.
    auto tp_count = [&](const UnitCoord& c) {
      named_bar_sync(1, Cfg::EPI_THREADS);
      if (ew == 0 && lane == 0) {
        // Release (system scope): the pushes ordered before this by the
        // barrier are visible to whoever acquires the count; acquire: the
        // other ranks' pushes are visible to us.
        unsigned long long* cnt = p.tp_counters[tp_owner(c)] + 2 + tp_wtile(c);
        const bool last = atom_add_acq_rel_sys(cnt, 1ull) == static_cast<unsigned long long>(p.tp_world - 1);
        // Reset for the next call: no rank counts on this tile again before
        // it has seen this tile delivered (its kernel waits for that).
        if (last) st_relaxed_sys(cnt, 0ull);
        *last_flag = last;
      }
      named_bar_sync(1, Cfg::EPI_THREADS);
      return *last_flag != 0;
    };
    // bf16 of v[0 .. n) (tile columns j0 ..) of row r / weight row r into every rank's output.
    auto tp_store = [&](int r, int col0, int j0, const float* v, int n) {
      for (int q = 0; q < p.tp_world; ++q) {
        if constexpr (!SWAP) {
          // Row r, 16-byte pieces (N and the row stride are multiples of 8,
          // outputs 16-byte aligned).
          __nv_bfloat16* o = p.tp_out[q] + int64_t(r) * p.tp_ldo + col0 + j0;
          for (int j = 0; j < n; j += 8)
            if (col0 + j0 + j < p.N)
              *reinterpret_cast<uint4*>(o + j) =
                  make_uint4(bf16x2_bits(v[j], v[j + 1]), bf16x2_bits(v[j + 2], v[j + 3]),
                             bf16x2_bits(v[j + 4], v[j + 5]), bf16x2_bits(v[j + 6], v[j + 7]));
        } else {
          // Weight row r is output column r; token col0 + j is an output row.
          __nv_bfloat16* o = p.tp_out[q] + r;
          for (int j = 0; j < n; ++j)
            if (col0 + j0 + j < p.M) o[int64_t(col0 + j0 + j) * p.tp_ldo] = __float2bfloat16_rn(v[j]);
        }
      }
    };
    // After the stores of a delivered tile (every thread's, by the barrier):
    // one more on every rank's delivery count.
    auto tp_delivered = [&]() {
      named_bar_sync(1, Cfg::EPI_THREADS);
      if (ew == 0 && lane == 0)
        for (int q = 0; q < p.tp_world; ++q) red_add_release_sys(p.tp_counters[q], 1ull);
    };
    // The sum of tile c's partials in rank order from zero, rounded once to
    // bf16 and delivered.  Full width, in this thread's accumulators.
    auto tp_sum_full = [&](const UnitCoord& c, int r, bool row_ok, bool cols_ok, int col0, float (&accum)[COLS],
                           bool ok) {
      if (row_ok && cols_ok && ok) {
#pragma unroll
        for (int j = 0; j < COLS; ++j) accum[j] = 0.f;
        for (int s = 0; s < p.tp_world; ++s) {
          const float* w = tp_slots(c) + s * tp_rank_stride;
#pragma unroll
          for (int j = 0; j < COLS; ++j) accum[j] += __ldcg(w + tp_col(j) * 128);
        }
        tp_store(r, col0, 0, accum, COLS);
      }
      tp_delivered();
    };
    // The same for a tile handed over earlier, while the accumulators hold
    // a newer tile: 32 columns at a time.
    auto tp_sum_chunked = [&](const UnitCoord& c, bool ok) {
      const int r = c.tr * Cfg::TILE_M + row_off + row;
      const int col0 = c.tc * BN + g * COLS;
      if (r < rows_total && col0 < (SWAP ? p.M : p.N) && ok) {
        constexpr int CH = COLS < 32 ? COLS : 32;
#pragma unroll 1
        for (int j0 = 0; j0 < COLS; j0 += CH) {
          float t[CH];
#pragma unroll
          for (int j = 0; j < CH; ++j) t[j] = 0.f;
          for (int s = 0; s < p.tp_world; ++s) {
            const float* w = tp_slots(c) + s * tp_rank_stride;
#pragma unroll
            for (int j = 0; j < CH; ++j) t[j] += __ldcg(w + tp_col(j0 + j) * 128);
          }
          tp_store(r, col0, j0, t, CH);
        }
      }
      tp_delivered();
    };
    // A tile of another rank is counted only at the end of this CTA's next
    // tile (or of the kernel): its pushes cross NVLink meanwhile, so the
    // release of the count does not wait for them.  A rank's own tiles are
    // counted at once (local pushes, and usually the completing arrival).
    UnitCoord tp_pending{};
    bool tp_has_pending = false;
    auto tp_flush = [&](bool ok) {
      if (tp_has_pending && tp_count(tp_pending)) tp_sum_chunked(tp_pending, ok);
      tp_has_pending = false;
    };

    int next_seq = 0;  // position of the next unit's first K block in the CTA's sequence
    for (int u = u0; any_unit && unit_valid(p, u, sid);) {
      const UnitCoord c = c_next;
      u = next_unit(p, u, c, scount);
      next_seq += c.kt1 - c.kt0;
      const ScaleSrc src = scale_src(c);
      const bool more = unit_valid(p, u, sid);
      if (more) {
        c_next = unit_coord(p, u, sid);
        prefetch_unit(c_next, na, na2, nb);
      }
      const int row0 = c.tr * Cfg::TILE_M + row_off;       // this CTA's first row of the tile
      const int r = row0 + row;                             // this thread's MMA row
      const bool row_ok = r < rows_total;
      const bool warp_rows = row0 + 32 * quarter < rows_total;  // warp-uniform
      const int col0 = c.tc * BN + g * COLS;                // first MMA column of this thread
      const int cols_total = SWAP ? p.M : p.N;
      const bool cols_ok = col0 < cols_total;               // warp-uniform
      const bool work = warp_rows && cols_ok;

      float accum[COLS];
#pragma unroll
      for (int j = 0; j < COLS; ++j) accum[j] = 0.f;

      for (int kt_base = c.kt0; kt_base < c.kt1; kt_base += PF) {
#pragma unroll
        for (int j = 0; j < PF; ++j) {
          const int kt = kt_base + j;
          if (kt < c.kt1) {
            float sa_v = pa[j], sb_v = pb[j];
            float sa2_v = 0.f;
            if constexpr (SWAP && BN > 32) sa2_v = pa2[j];
            if (kt + PF < c.kt1) load_scales(src, kt + PF, pa[j], pa2[j], pb[j]);
            if constexpr (FUSE) {  // the token scales quantize_unit wrote for this K block
              const uint32_t sl = s_act_scales + uint32_t((kt - c.kt0) * BN) * 4u;
              sa_v = lane < BN ? ld_shared_f32(sl + uint32_t(lane) * 4u) : 0.f;
              if constexpr (BN > 32) sa2_v = ld_shared_f32(sl + uint32_t(32 + lane) * 4u);
            }
            // This warp's release of TMEM buffer acc's column block h.
            auto release = [&](int h) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) {
                if constexpr (PAIR) mbar_arrive_cluster(leader_bar(acc_empty(acc, h)));
                else mbar_arrive(acc_empty(acc, h));
              }
            };
            if constexpr (!SWAP) {
              // Warpgroup g promotes column block g.  One scale per thread:
              // sa[row] * sb[block], as the reference forms it; 32-column
              // chunks loaded two at a time, promoted with packed fmas (each
              // lane of fma.rn.f32x2 rounds like fmaf).  The buffer's block
              // goes back to the MMA issuer as soon as its last chunks are in
              // registers, before their fmas (3% on the 256 x 256 tiles).
              ok = mbar_wait(acc_full(acc, g), acc_phase, abort_flag, kWaitAccFull) && ok;
              tc_fence_after();
              bool released = false;
              if (work) {
                const uint32_t t = t_lane + uint32_t(acc * BN + g * COLS);
                const float scale = sa_v * sb_v;
#pragma unroll
                for (int ch = 0; ch < COLS / 32; ch += 2) {
                  uint32_t r0[32], r1[32];
                  tmem_ld32_async(t + 32 * ch, r0);
                  if (ch + 1 < COLS / 32) tmem_ld32_async(t + 32 * (ch + 1), r1);
                  tmem_wait_ld();
                  if (ch + 2 >= COLS / 32) {  // the block's last columns are in registers: buffer free
                    release(g);
                    released = true;
                  }
#pragma unroll
                  for (int i = 0; i < 32; i += 2)
                    fma2(accum[32 * ch + i], accum[32 * ch + i + 1], __uint_as_float(r0[i]),
                         __uint_as_float(r0[i + 1]), scale, scale);
                  if (ch + 1 < COLS / 32) {
#pragma unroll
                    for (int i = 0; i < 32; i += 2)
                      fma2(accum[32 * (ch + 1) + i], accum[32 * (ch + 1) + i + 1], __uint_as_float(r1[i]),
                           __uint_as_float(r1[i + 1]), scale, scale);
                  }
                }
              }
              if (!released) release(g);
            } else {
              ok = mbar_wait(acc_full(acc, 0), acc_phase, abort_flag, kWaitAccFull) && ok;
              tc_fence_after();
              if (work) {
                const uint32_t t = t_lane + uint32_t(acc * BN);
                constexpr int CH = BN < 32 ? BN : 32;
#pragma unroll
                for (int ch = 0; ch < BN / CH; ++ch) {
                  float part[CH];
                  tmem_ld<CH>(t + CH * ch, part);
                  const float src_s = ch == 0 ? sa_v : sa2_v;
#pragma unroll
                  for (int i = 0; i < CH; i += 2) {
                    const float s0 = __shfl_sync(0xffffffffu, src_s, i) * sb_v;
                    const float s1 = __shfl_sync(0xffffffffu, src_s, i + 1) * sb_v;
                    fma2(accum[CH * ch + i], accum[CH * ch + i + 1], part[i], part[i + 1], s0, s1);
                  }
                }
              }
              release(0);
            }
            if (++acc == ACC_BUFS) {
              acc = 0;
              acc_phase ^= 1u;
            }
          }
        }
      }

      // The next unit's scales move into the ring; FUSE quantizes the next
      // unit now, ahead of this unit's split-K hand-off and store (all of
      // this unit's MMAs are done: every K block's partial has been read,
      // and every epilogue thread is past its scales).
      if (more) {
#pragma unroll
        for (int j = 0; j < PF; ++j) {
          pa[j] = na[j];
          pa2[j] = na2[j];
          pb[j] = nb[j];
        }
        if constexpr (FUSE) {
          named_bar_sync(1, Cfg::EPI_THREADS);
          publish_unit(c_next, next_seq);
        }
      }

      bool store = work;
      bool tile_whole = true;  // this CTA holds the tile's sum over its K range
      if (c.pieces > 1) {
        // Deterministic split-K: publish this split's partial, count arrivals;
        // the last CTA of the tile sums all partials in split order.
        // Partials per 128-row tile half (a pair's CTAs hand off separately).
        const int wtile = PAIR ? c.tile * 2 + int(rank) : c.tile;
        const int64_t split_stride = int64_t(p.tiles) * (PAIR ? 2 : 1) * (128 * BN);
        float* ws_tile = p.workspace + int64_t(wtile) * (128 * BN);
        if (row_ok && cols_ok && ok) {
          if constexpr (!SWAP) {
            float* w = ws_tile + c.split * split_stride + row * BN + g * COLS;
#pragma unroll
            for (int j = 0; j < COLS; j += 4)
              __stcg(reinterpret_cast<float4*>(w + j),
                     make_float4(accum[j], accum[j + 1], accum[j + 2], accum[j + 3]));
          } else {
            float* w = ws_tile + c.split * split_stride + row;
#pragma unroll
            for (int j = 0; j < COLS; ++j) __stcg(w + j * 128, accum[j]);
          }
        }
        // Every epilogue thread's partial is ordered before the counter
        // update by the barrier and lane 0's gpu-scope release; its acquire
        // makes the other parts' partials visible to the last arriver.
        named_bar_sync(1, Cfg::EPI_THREADS);
        if (ew == 0 && lane == 0)
          *last_flag = atom_add_acq_rel_gpu(p.counters + wtile, 1) == c.pieces - 1;
        named_bar_sync(1, Cfg::EPI_THREADS);
        const bool last = *last_flag != 0;
        store = store && last;
        tile_whole = last;
        if (last) {
          if (row_ok && cols_ok) {
            // Sum every split's partial (this CTA's own included, as written
            // above) in split order starting from zero, like the reference:
            // one pass per split with all of a split's loads in flight.
#pragma unroll
            for (int j = 0; j < COLS; ++j) accum[j] = 0.f;
            for (int s = 0; s < c.pieces; ++s) {
              if constexpr (!SWAP) {
                const float* w = ws_tile + s * split_stride + row * BN + g * COLS;
#pragma unroll
                for (int j = 0; j < COLS; j += 4) {
                  const float4 t = __ldcg(reinterpret_cast<const float4*>(w + j));
                  accum[j] += t.x;
                  accum[j + 1] += t.y;
                  accum[j + 2] += t.z;
                  accum[j + 3] += t.w;
                }
              } else {
                const float* w = ws_tile + s * split_stride + row;
#pragma unroll
                for (int j = 0; j < COLS; ++j) accum[j] += __ldcg(w + j * 128);
              }
            }
          }
          if (ew == 0 && lane == 0) p.counters[wtile] = 0;  // ready for the next launch
        }
      }

      if constexpr (Cfg::TP) {
        if (tile_whole) {  // CTA-uniform
          tp_flush(ok);    // the previous tile of another rank, before this tile's pushes
          tp_push(c, row_ok, cols_ok, accum, ok);
          if (tp_owner(c) == p.tp_rank) {
            if (tp_count(c)) tp_sum_full(c, r, row_ok, cols_ok, col0, accum, ok);
          } else {
            tp_pending = c;
            tp_has_pending = true;
          }
        }
      } else if (store && ok) {
        if constexpr (!SWAP) {
          // bf16 rows -> [32 x 32] chunks, 64-byte swizzle, two buffers in
          // turn so one chunk's TMA store overlaps the next chunk's writes.
#pragma unroll
          for (int ch = 0; ch < COLS / 32; ++ch) {
            const int col = col0 + 32 * ch;
            if (col >= p.N) break;
            const uint32_t buf = out_buf + uint32_t(out_chunk) * 2048u;
            if (lane == 0) bulk_wait_read1();  // the store that last read this buffer is done
            __syncwarp();
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const float* a = accum + 32 * ch + 8 * v;
              const uint32_t dst = buf + uint32_t(lane) * 64u + uint32_t((v ^ ((lane >> 1) & 3)) * 16);
              st_shared_v4(dst, bf16x2_bits(a[0], a[1]), bf16x2_bits(a[2], a[3]), bf16x2_bits(a[4], a[5]),
                           bf16x2_bits(a[6], a[7]));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&p.map_c, col, row0 + 32 * quarter, buf);
              bulk_commit();
            }
            out_chunk ^= 1;
          }
        } else {
          // [BN tokens x 32 weight rows] bf16, row-major: TMA box {32, BN}.
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < COLS; ++j)
            st_shared_b16(out_buf + uint32_t(j) * 64u + uint32_t(lane) * 2u,
                          __bfloat16_as_ushort(__float2bfloat16_rn(accum[j])));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&p.map_c, c.tr * 128 + 32 * quarter, c.tc * BN, out_buf);
            bulk_commit();
          }
        }
      }
    }
    if constexpr (Cfg::TP) tp_flush(ok);
    if (Cfg::TP && blockIdx.x == 0 && ew == 0 && lane == 0) {
      // This rank's output is complete once every tile half has been
      // delivered (by whichever rank summed it): counter [0] reaches the
      // tiles of all calls so far, counter [1] (written only here) plus
      // this call's.  The kernel ends after that.
      unsigned long long* mine = p.tp_counters[p.tp_rank];
      const unsigned long long target = mine[1] + static_cast<unsigned long long>(p.tiles) * (PAIR ? 2 : 1);
      const uint64_t t0 = globaltimer();
      while (p.tp_wait && ld_acquire_sys(mine) < target) {
        if (*abort_flag || globaltimer() - t0 > kWaitTimeoutNs) {
          record_status((0x5Bull << 56) | (uint64_t(kWaitTpDelivered) << 32) | (uint64_t(blockIdx.x) << 8) |
                        uint64_t(warp));
          break;
        }
        __nanosleep(64);
      }
      mine[1] = target;
    }
    if (lane == 0) bulk_wait0();  // stores complete before the CTA retires
  }

  tc_fence_before();
  // A pair: the leader's MMAs (which read this CTA's tiles and write its
  // TMEM) and both CTAs' remote arrivals are over before either frees
  // TMEM or exits.
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace bfp8
