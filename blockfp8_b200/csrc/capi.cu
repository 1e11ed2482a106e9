// Host side of blockfp8_b200: configurations, the planner, tensor maps,
// launches and the C ABI declared in include/blockfp8_b200.h.
//
// Counterparts in the reference (simon-jd/blockfp8): csrc/gemm_sm89.cu
// (configurations :71-114, plan lookup :159-224, split sizing :250-279,
// launch :281-286) and csrc/quant_sm89.cu:66-71.  The tables, the cost model
// and the launch plumbing here are written for B200: 148 SMs, one
// persistent CTA per SM, tensor maps for TMA.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "blockfp8_b200.h"

#include <algorithm>
#include <vector>

#include "gemm_kernel.cuh"
#include "probes.cuh"
#include "producers.cuh"
#include "quantize.cuh"
#include "stream_gemm.cuh"

namespace bfp8 {
namespace {

thread_local std::string t_last_error;

int fail(int code, const std::string& msg) {
  t_last_error = "blockfp8: " + msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  cudaGetLastError();  // not sticky: do not leave it for the caller's next check
  return fail(BFP8_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int cdiv(int a, int b) { return (a + b - 1) / b; }

// ---- compiled configurations ---------------------------------------------------

struct ConfigEntry {
  const char* name;
  int bn, stages, threads, smem;
  bool swap;  // MMA rows are weight rows, columns are tokens (decode)
  int bm;     // MMA rows of a tile: 128, or 256 for a CTA pair
  bool pair;  // a cluster of two CTAs per tile (cta_group::2)
  const void* kernel;
  void (*launch)(const GemmParams&, int grid, cudaStream_t);
  // Swapped configurations also come with the activation quantization done
  // inside the kernel (bf16 in), used by fused plans.
  const void* kernel_fused = nullptr;
  void (*launch_fused)(const GemmParams&, int grid, cudaStream_t) = nullptr;
  int smem_fused = 0, threads_fused = 0;
  // The row-parallel twins (bfp8_launch_gemm_tp) of both kernels.
  const void* kernel_tp = nullptr;
  void (*launch_tp)(const GemmParams&, int grid, cudaStream_t) = nullptr;
  const void* kernel_fused_tp = nullptr;
  void (*launch_fused_tp)(const GemmParams&, int grid, cudaStream_t) = nullptr;
  int act_kb = 0;  // K blocks of one unit the in-kernel variant keeps resident
  // Weight-streaming configurations (stream_gemm.cuh): at most max_m tokens,
  // stream-K over the SMs, activations resident; no row-parallel twin.
  bool stream = false;
  int max_m = 0;
  const void* kernel_stream = nullptr;  // [0] quantized activations, [1] bf16 (in-kernel quantization)
  const void* kernel_stream_q = nullptr;
  void (*launch_stream)(const StreamParams&, int grid, int smem, bool pdl, cudaStream_t) = nullptr;
  void (*launch_stream_q)(const StreamParams&, int grid, int smem, bool pdl, cudaStream_t) = nullptr;
};

template <class Cfg>
void launch_cfg(const GemmParams& gp, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (!Cfg::FUSE) {  // these variants wait before reading activations (in-kernel quantization does not)
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n++].val.programmaticStreamSerializationAllowed = 1;
  }
  if (Cfg::PAIR) {  // CTA pairs: clusters of two along x
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 2;
    attr[n].val.clusterDim.y = 1;
    attr[n++].val.clusterDim.z = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaLaunchKernelEx(&cfg, gemm_kernel<Cfg>, gp);
}

template <class Cfg>
ConfigEntry entry(const char* name) {
  ConfigEntry e{name, Cfg::BN, Cfg::STAGES, Cfg::THREADS, Cfg::SMEM_BYTES, Cfg::SWAP, Cfg::TILE_M, Cfg::PAIR,
                reinterpret_cast<const void*>(&gemm_kernel<Cfg>), &launch_cfg<Cfg>};
  e.kernel_tp = reinterpret_cast<const void*>(&gemm_kernel<WithTp<Cfg>>);
  e.launch_tp = &launch_cfg<WithTp<Cfg>>;
  return e;
}

template <class Cfg, class FusedCfg>
ConfigEntry entry_fused(const char* name) {
  ConfigEntry e = entry<Cfg>(name);
  e.kernel_fused = reinterpret_cast<const void*>(&gemm_kernel<FusedCfg>);
  e.launch_fused = &launch_cfg<FusedCfg>;
  e.smem_fused = FusedCfg::SMEM_BYTES;
  e.threads_fused = FusedCfg::THREADS;
  e.kernel_fused_tp = reinterpret_cast<const void*>(&gemm_kernel<WithTp<FusedCfg>>);
  e.launch_fused_tp = &launch_cfg<WithTp<FusedCfg>>;
  e.act_kb = FusedCfg::ACT_KB;
  return e;
}

template <class Cfg>
void launch_stream_cfg(const StreamParams& sp, int grid, int smem, bool pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, stream_kernel<Cfg>, sp);
}

template <int BN>
ConfigEntry entry_stream(const char* name) {
  using C = StreamCfg<BN, false>;
  using Q = StreamCfg<BN, true>;
  ConfigEntry e{name, BN, 0, C::THREADS, 0, true, 128, false, nullptr, nullptr};
  e.stream = true;
  e.max_m = BN;
  e.kernel_stream = reinterpret_cast<const void*>(&stream_kernel<C>);
  e.kernel_stream_q = reinterpret_cast<const void*>(&stream_kernel<Q>);
  e.launch_stream = &launch_stream_cfg<C>;
  e.launch_stream_q = &launch_stream_cfg<Q>;
  return e;
}

// Normal order: "m128n<BN>": 128 activation rows x BN weight rows per tile;
// "m256n256": 256 x 256 tiles on a CTA pair (cta_group::2, prefill).
// Swapped order: "w128t<BN>": 128 weight rows x BN tokens per tile (decode).
// Weight streaming: "w128d<BN>": the swapped order for at most BN tokens,
// every SM streaming an equal share of the weight tiles (stream_gemm.cuh).
//                        BN  stages  swapped
using Cfg256 = GemmCfg<256, 4, false>;
using Cfg128 = GemmCfg<128, 6, false>;
using Cfg64 = GemmCfg<64, 8, false>;
using CfgW16 = GemmCfg<16, 10, true>;
using CfgW32 = GemmCfg<32, 10, true>;
using CfgW64 = GemmCfg<64, 8, true>;
// ... quantizing in the kernel: the unit's B operand is resident (64 KB),
// the ring carries only weight tiles
using CfgW16Q = GemmCfg<16, 8, true, true>;
using CfgW32Q = GemmCfg<32, 8, true, true>;
using CfgW64Q = GemmCfg<64, 8, true, true>;
// ... a CTA pair: 32 KB per CTA per stage (its 128 A rows, half the B rows)
using CfgP256 = GemmCfg<256, 6, false, false, true>;

const ConfigEntry kConfigs[] = {
    entry<Cfg256>("m128n256s4"),
    entry<Cfg128>("m128n128s6"),
    entry<Cfg64>("m128n64s8"),
    entry_fused<CfgW16, CfgW16Q>("w128t16s10"),
    entry_fused<CfgW32, CfgW32Q>("w128t32s10"),
    entry_fused<CfgW64, CfgW64Q>("w128t64s8"),
    entry<CfgP256>("m256n256s6"),
    entry_stream<16>("w128d16"),
    entry_stream<32>("w128d32"),
    entry_stream<64>("w128d64"),
};
constexpr int kNumConfigs = int(sizeof(kConfigs) / sizeof(kConfigs[0]));
// The fused path (gemm_bf16) quantizes into the workspace, then runs the
// same GEMM kernels, so it has the same configurations.
constexpr int kNumFusedConfigs = kNumConfigs;

bool config_ok(int config) { return config >= 0 && config < kNumConfigs; }

// ---- per-device state -------------------------------------------------------------

constexpr int kMaxDevices = 64;

int current_device_sms(int* dev_out) {
  static std::atomic<int> sms[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (dev_out) *dev_out = dev;
  if (dev >= kMaxDevices) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
  }
  int n = sms[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    sms[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// The dynamic shared-memory limit is a per-device attribute of a kernel:
// set it on the first launch of each configuration on each device.
// Weight-streaming kernels size their shared memory per launch, up to this.
constexpr int kMaxSmem = 232448;

int ensure_smem_attr(int config, int dev, bool in_kernel_quant, bool tp = false) {
  static std::atomic<uint64_t> done[4][kNumConfigs] = {};
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  std::atomic<uint64_t>& d = done[(in_kernel_quant ? 1 : 0) + (tp ? 2 : 0)][config];
  if (bit && (d.load(std::memory_order_acquire) & bit)) return BFP8_OK;
  const ConfigEntry& e = kConfigs[config];
  const void* kernel = e.stream ? (in_kernel_quant ? e.kernel_stream_q : e.kernel_stream)
                                : in_kernel_quant ? (tp ? e.kernel_fused_tp : e.kernel_fused)
                                                  : (tp ? e.kernel_tp : e.kernel);
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         e.stream ? kMaxSmem : in_kernel_quant ? e.smem_fused : e.smem);
  if (err != cudaSuccess) return cuda_fail(err, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  if (e.stream) {  // two CTAs of up to 112 KB on one SM
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (err != cudaSuccess) return cuda_fail(err, "cudaFuncSetAttribute(PreferredSharedMemoryCarveout)");
  }
  d.fetch_or(bit, std::memory_order_release);
  return BFP8_OK;
}

// A plan's shape.  Round-robin split-K: `splits` parts of k_per_split K
// blocks per tile.  Stream-K (plan.splits < 0): sk_grid CTAs share the
// sk_work = tiles * k_tiles K blocks evenly; k_per_split is then the longest
// unit and `splits` the most parts any tile is cut into.
struct Derived {
  int tiles_r, tiles_c, tiles, k_tiles, k_per_split, splits;
  int sk_grid = 0;
  int64_t sk_work = 0;
};
Derived derive(const bfp8_gemm_problem& p, const bfp8_plan& plan);

// Plans that ask for quantization inside the GEMM, of swapped configurations
// whose units fit the resident operand, quantize in the GEMM kernel; other
// fused plans run the quantization kernel into the workspace first (same
// results either way).
bool quantizes_in_kernel(const bfp8_gemm_problem& p, const bfp8_plan& plan) {
  const ConfigEntry& e = kConfigs[plan.config];
  if (e.stream) return plan.fused == BFP8_FUSED_IN_GEMM;
  return plan.fused == BFP8_FUSED_IN_GEMM && e.launch_fused != nullptr &&
         derive(p, plan).k_per_split <= e.act_kb;
}

// ---- tensor maps --------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

int make_map(CUtensorMap* map, CUtensorMapDataType dtype, const void* ptr, uint64_t inner,
             uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
             CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return fail(BFP8_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estrides[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estrides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BFP8_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return BFP8_OK;
}

// ---- plan tables (B200) ----------------------------------------------------------

struct TableEntry {
  int n, k, m, config, splits;
};
// Winners of the autotuning sweep on a B200 (blockfp8_b200/autotune.py).
const TableEntry kPlanTable[] = {
#include "plan_table.inc"
    {0, 0, 0, 0, 0}};
constexpr int kPlanEntries = int(sizeof(kPlanTable) / sizeof(kPlanTable[0])) - 1;

// Fused plans (bf16 in): the faster of quantization kernel + GEMM and
// quantization inside the GEMM, with its own configuration and splits,
// where the sweep timed both (decode sizes).
struct FusedTableEntry {
  int n, k, m, config, splits, mode;
};
const FusedTableEntry kFusedPlanTable[] = {
#include "fused_plan_table.inc"
    {0, 0, 0, 0, 0, 0}};
constexpr int kFusedPlanEntries = int(sizeof(kFusedPlanTable) / sizeof(kFusedPlanTable[0])) - 1;

// The entry for this (N, K) with the smallest tabulated M >= M, else the
// largest (the reference's lookup rule, csrc/gemm_sm89.cu:158-169).
template <class E>
const E* lookup(const E* table, int n_entries, int M, int N, int K) {
  const E* best = nullptr;
  for (int i = 0; i < n_entries; ++i) {
    const E& t = table[i];
    if (t.n != N || t.k != K || !config_ok(t.config)) continue;
    const bool better =
        !best || (t.m >= M ? (best->m < M || t.m < best->m) : (best->m < M && t.m > best->m));
    if (better) best = &t;
  }
  return best;
}

// Cost model of one plan on B200, in nanoseconds, for untabulated shapes and
// for the balanced choice between tabulated plans.  A persistent CTA per SM
// runs ceil(units / SMs) units of k_per_split K blocks; a K block costs the
// larger of its MMA time (4 MMAs of 128 x BN x 32 at 8192 e4m3 MACs per SM
// clock) and its operand bytes at the SM's share of HBM bandwidth; split-K
// adds the fp32 partial round trip of the valid rows.  Stream-K (splits < 0)
// is one wave of -splits CTAs with ceil(W / CTAs) K blocks each and up to
// two units (and partial round trips) per CTA.
double plan_cost_ns(int M, int N, int K, int num_sms, int config, int splits) {
  const ConfigEntry& e = kConfigs[config];
  if (e.stream) {  // the weights at HBM rate over the CTAs that stream them, plus fill and tail
    if (M > e.max_m) return 1e300;
    const int64_t work = int64_t(cdiv(N, 128)) * cdiv(K, 128);
    const int64_t g = splits < 0 ? std::min<int64_t>(-int64_t(splits), work) : std::min<int64_t>(work, int64_t(cdiv(N, 128)) * splits);
    const double share = double(std::min<int64_t>(g, num_sms)) / num_sms;
    return double(N) * K / (6500.0 * std::max(share, 1e-3)) + 3000.0;
  }
  const int k_tiles = cdiv(K, 128);
  const int rows_total = e.swap ? N : M, cols_total = e.swap ? M : N;
  const int tiles_r = cdiv(rows_total, e.bm), tiles_c = cdiv(cols_total, e.bn);
  const int ctas_per_unit = e.pair ? 2 : 1;
  const int slots = std::max(1, num_sms / ctas_per_unit);  // units in flight at once
  int per, real_splits;
  int64_t waves;
  int active;
  if (splits < 0) {
    if (e.pair) return 1e300;  // no stream-K schedule for CTA pairs
    const int64_t work = int64_t(tiles_r) * tiles_c * k_tiles;
    const int64_t g = std::max<int64_t>(1, std::min<int64_t>(-int64_t(splits), work));
    per = int((work + g - 1) / g);
    real_splits = per < k_tiles ? 2 : 1;  // a partial round trip in most units
    waves = per < k_tiles ? 2 : (per + k_tiles - 1) / k_tiles;  // units per CTA
    active = int(g);
    per = int((work + g - 1) / g / waves);  // K blocks per unit, on average
  } else {
    per = cdiv(k_tiles, std::max(1, std::min(splits, k_tiles)));
    real_splits = cdiv(k_tiles, per);
    const int64_t units = int64_t(tiles_r) * tiles_c * real_splits;
    waves = (units + slots - 1) / slots;
    active = int(std::min<int64_t>(units, slots)) * ctas_per_unit;
  }
  const double clk_ghz = 1.8;
  const double mma_ns = 2.0 * e.bn / clk_ghz;
  // A CTA's K block: its 128 rows of A and its share of the B rows.
  const int rows = std::min(rows_total, 128);
  const double bytes = double(rows) * 128 + double(std::min(cols_total, e.bn)) * 128 / ctas_per_unit;
  const double hbm_gbs = 6500.0, l2_sm_gbs = 120.0;
  const double sm_gbs = std::min(l2_sm_gbs, hbm_gbs / active);
  const double load_ns = bytes / sm_gbs;
  // The promotion of a K block: each warp that owns valid rows loads its
  // columns from TMEM in 32-column chunks, one after another.
  const double epi_ns = 40.0 + 60.0 * std::max(1, std::min(e.bn, e.swap ? e.bn : 128) / 32);
  double t = double(waves) * per * std::max(std::max(mma_ns, load_ns), epi_ns);
  const double tile_out = double(rows) * e.bn;
  t += double(waves) * tile_out * 2 / (hbm_gbs / active) * 1.0;  // bf16 store
  if (real_splits > 1) t += double(waves) * tile_out * 4 * 2 / sm_gbs + 600.0;
  return t + 2000.0;  // launch and pipeline fill
}

// Up to 32 tokens the swapped (decode) configurations won 25 of the 27
// tuned shapes on B200, and the cost model underrates their advantage, so
// untabulated shapes there only consider them.
constexpr int kSwappedOnlyM = 32;

bfp8_plan heuristic_plan(int M, int N, int K, int num_sms, bool fused) {
  bfp8_plan best{1, 1, fused ? 1 : 0};
  double best_t = 1e300;
  const int k_tiles = cdiv(K, 128);
  for (int config = 0; config < kNumConfigs; ++config) {
    if (kConfigs[config].stream) continue;  // chosen by stream_plan, not by this model
    if (M <= kSwappedOnlyM && !kConfigs[config].swap) continue;
    for (int splits = 0; splits <= std::min(k_tiles, 16); ++splits) {
      if (splits == 0) {  // stream-K over every SM
        const double t = plan_cost_ns(M, N, K, num_sms, config, -num_sms);
        if (t < best_t * 0.999) {
          best_t = t;
          best = {config, -num_sms, fused ? 1 : 0};
        }
        continue;
      }
      const int per = cdiv(k_tiles, splits);
      if (cdiv(k_tiles, per) != splits) continue;  // same as a smaller split count
      const double t = plan_cost_ns(M, N, K, num_sms, config, splits);
      if (t < best_t * 0.999) {
        best_t = t;
        best = {config, splits, fused ? 1 : 0};
      }
    }
  }
  return best;
}

// Among the plans tabulated for this shape at M / 4 .. 4 M, the one the cost
// model rates fastest at this M; ties keep the entry above (the reference's
// balanced_entry, csrc/gemm_sm89.cu:190-224, with the B200 cost model in place
// of its busiest-SM work count).
const TableEntry* balanced_entry(const TableEntry* above, int M, int N, int K, int num_sms) {
  if (M < 256 || above->m == M) return above;
  const TableEntry* best = above;
  double best_t = plan_cost_ns(M, N, K, num_sms, above->config, above->splits);
  for (int i = 0; i < kPlanEntries; ++i) {
    const TableEntry& t = kPlanTable[i];
    if (t.n != N || t.k != K || !config_ok(t.config)) continue;
    if (4 * int64_t(t.m) < M || t.m > 4 * int64_t(M)) continue;
    const double c = plan_cost_ns(M, N, K, num_sms, t.config, t.splits);
    if (c < best_t * 0.98) {
      best = &t;
      best_t = c;
    }
  }
  return best;
}

Derived derive(const bfp8_gemm_problem& p, const bfp8_plan& plan) {
  const ConfigEntry& e = kConfigs[plan.config];
  Derived d;
  d.tiles_r = cdiv(e.swap ? p.N : p.M, e.bm);
  d.tiles_c = e.stream ? 1 : cdiv(e.swap ? p.M : p.N, e.bn);
  d.tiles = d.tiles_r * d.tiles_c;
  d.k_tiles = cdiv(p.K, 128);
  if (e.stream) {
    // Weight streaming: always one contiguous range of the tiles' K blocks
    // per CTA; `splits` K splits per tile ask for tiles * splits CTAs,
    // negative splits for -splits CTAs.
    const int64_t W = int64_t(d.tiles) * d.k_tiles;
    const int64_t want = plan.splits > 0 ? int64_t(d.tiles) * std::min(plan.splits, d.k_tiles) : -int64_t(plan.splits);
    Derived s = d;
    const int64_t G = std::max<int64_t>(1, std::min<int64_t>(want, W));
    s.sk_grid = int(G);
    s.sk_work = W;
    s.k_per_split = int((W + G - 1) / G);  // the longest range (positions)
    auto starts_upto = [&](int64_t x) { return std::min<int64_t>(G, ((x + 1) * G + W - 1) / W); };
    int most = 1;
    for (int t = 0; t < d.tiles; ++t) {
      const int64_t t0 = int64_t(t) * d.k_tiles;
      most = std::max(most, int(starts_upto(t0 + d.k_tiles - 1) - starts_upto(t0) + 1));
    }
    s.splits = most;
    return s;
  }
  if (plan.splits < 0) {
    // Stream-K: CTA b takes K-block positions [W b / G, W (b + 1) / G); the
    // CTAs starting at or before position x number min(G, ceil((x + 1) G / W)).
    const int64_t W = int64_t(d.tiles) * d.k_tiles;
    const int64_t G = std::max<int64_t>(1, std::min<int64_t>(-int64_t(plan.splits), W));
    d.sk_grid = int(G);
    d.sk_work = W;
    d.k_per_split = int(std::min<int64_t>(d.k_tiles, (W + G - 1) / G));
    auto starts_upto = [&](int64_t x) { return std::min<int64_t>(G, ((x + 1) * G + W - 1) / W); };
    int most = 1;
    for (int t = 0; t < d.tiles; ++t) {
      const int64_t t0 = int64_t(t) * d.k_tiles;
      most = std::max(most, int(starts_upto(t0 + d.k_tiles - 1) - starts_upto(t0) + 1));
    }
    d.splits = most;
    return d;
  }
  const int splits = std::max(1, std::min(plan.splits, d.k_tiles));
  d.k_per_split = cdiv(d.k_tiles, splits);
  d.splits = cdiv(d.k_tiles, d.k_per_split);  // no empty splits
  return d;
}

int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

// Fused plans: quantized activations [M, K] then M-major scales [kb, M].
int64_t fused_front_bytes(const bfp8_gemm_problem& p) {
  const int64_t kb = cdiv(p.K, 128);
  return align256(int64_t(p.M) * p.K) + align256(kb * p.M * 4);
}

int64_t splitk_bytes(const bfp8_gemm_problem& p, const bfp8_plan& plan) {
  const Derived d = derive(p, plan);
  if (d.splits == 1) return 0;
  const ConfigEntry& e = kConfigs[plan.config];
  // weight streaming: [tiles][parts][128 rows][M tokens rounded up to 4] fp32
  if (e.stream) return int64_t(d.tiles) * d.splits * 128 * ((p.M + 3) & ~3) * int64_t(sizeof(float));
  // one fp32 partial per 128-row tile (a CTA pair's tile has two)
  return int64_t(d.splits) * d.tiles * (e.bm / 128) * 128 * e.bn * int64_t(sizeof(float));
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int check_problem(const bfp8_gemm_problem& p, bool fused) {
  if (p.M < 0 || p.N <= 0 || p.K <= 0) return fail(BFP8_EINVAL, "bad shapes (M >= 0, N > 0, K > 0)");
  if (p.K % 16 != 0) return fail(BFP8_EINVAL, "K must be a positive multiple of 16");
  if (p.N % 8 != 0) return fail(BFP8_EINVAL, "N must be a positive multiple of 8");
  if (p.M == 0) return BFP8_OK;
  if (!p.a || !p.b || !p.c || !p.sb || (!fused && !p.sa)) return fail(BFP8_EINVAL, "null operand pointer");
  if (!aligned16(p.a) || !aligned16(p.b) || !aligned16(p.c))
    return fail(BFP8_EINVAL, "a, b and c must be 16-byte aligned");
  const int64_t a_elem = fused ? 2 : 1;
  if (p.lda < p.K || (p.lda * a_elem) % 16 != 0)
    return fail(BFP8_EINVAL, "a must be row-major with 16-byte aligned rows");
  if (p.ldb < p.K || p.ldb % 16 != 0) return fail(BFP8_EINVAL, "b must be row-major with 16-element aligned rows");
  if (p.ldc < p.N || p.ldc % 8 != 0) return fail(BFP8_EINVAL, "c must be row-major with 8-element aligned rows");
  if (fused && !(p.eps > 0.f)) return fail(BFP8_EINVAL, "eps must be positive");
  return BFP8_OK;
}

// Weight tiles (and their scales) may be requested before the previous
// kernel of the stream has finished (programmatic dependent launch); on by
// default, see bfp8_set_weight_prefetch.
std::atomic<int> g_weight_prefetch{1};

// Every launch carries the programmatic-serialization attribute, so that it
// can start while the previous kernel of the stream finishes; each kernel
// waits (griddepcontrol.wait) before it reads anything a previous kernel
// may write and before it writes anything.
void set_pdl(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr) {
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
}

int launch_quant(const QuantParams& qp, cudaStream_t stream, int num_sms) {
  // Four groups per task unless that leaves fewer tasks than two per SM.
  const bool small = int64_t(cdiv(qp.M, kQuantRows)) * cdiv(qp.kb, kQuantGroups) < 2 * int64_t(num_sms);
  const int64_t tasks = int64_t(cdiv(qp.M, kQuantRows)) * cdiv(qp.kb, small ? 1 : kQuantGroups);
  if (tasks == 0) return BFP8_OK;
  if (tasks >= (int64_t(1) << 31)) return fail(BFP8_EINVAL, "too many rows x K groups for one quantization launch");
  // Eight CTAs per SM: more loads in flight per SM than the four that are
  // resident at once, so the CTAs of the second wave start as the first ones
  // drain (measured faster than one resident wave at M = 8192, K = 4096).
  const int grid = int(std::min<int64_t>(tasks, int64_t(num_sms) * 8));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kQuantThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  set_pdl(cfg, attr);
  if (small) cudaLaunchKernelEx(&cfg, quantize_kernel<1>, qp);
  else cudaLaunchKernelEx(&cfg, quantize_kernel<kQuantGroups>, qp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "quantize kernel launch");
  return BFP8_OK;
}

// ---- fixed scratch for callers that cannot allocate --------------------------
// One array per device that loads this library, held until the process
// exits: the first BFP8_STATIC_COUNTER_BYTES hold split-K arrival counters,
// the rest the workspace (split-K partials, the fused path's quantized
// activations).  Host code must not use the array's name as a device
// address; static_scratch() looks the address up per device.
static __device__ __align__(256) unsigned char g_static_scratch[BFP8_STATIC_SCRATCH_BYTES];

// Device address of g_static_scratch on the current device, looked up once
// per device (cudaGetSymbolAddress, with that device current) and cached.
int static_scratch(int dev, unsigned char** out) {
  static std::mutex mu;
  static unsigned char* ptrs[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) return fail(BFP8_EINVAL, "device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    ptrs[dev] = static_cast<unsigned char*>(ptr);
  }
  *out = ptrs[dev];
  return BFP8_OK;
}

// Decode batches (up to kStreamMaxM tokens) go to the weight-streaming
// configurations: the smallest token tile that holds M, stream-K over every
// SM.  The linear path puts the quantization kernel ahead of it, which lets
// the streaming kernel load its first weight stages while the quantizer
// runs.  Quantizing inside the streaming kernel (plan.fused = 2, kept and
// tested) is faster only when linears run back to back with nothing between
// them, up to 2 tokens; with the other kernels of a model between the calls
// it is 0.3-1.6 us slower per linear on B200, so the plan never picks it.
constexpr int kStreamMaxM = 32;
constexpr int kStreamInGemmMaxM = 0;

bfp8_plan stream_plan(int M, int N, int K, int num_sms) {
  (void)N;
  (void)K;
  int best = -1;
  for (int c = 0; c < kNumConfigs; ++c)
    if (kConfigs[c].stream && kConfigs[c].max_m >= M && (best < 0 || kConfigs[c].max_m < kConfigs[best].max_m))
      best = c;
  return {best, -std::max(1, num_sms), 0};
}

}  // namespace
}  // namespace bfp8

using namespace bfp8;

extern "C" {

int bfp8_abi_version(void) { return 1; }

const char* bfp8_last_error(void) { return t_last_error.c_str(); }

int bfp8_num_configs(void) { return kNumConfigs; }
int bfp8_num_fused_configs(void) { return kNumFusedConfigs; }

const char* bfp8_config_name(int config) { return config_ok(config) ? kConfigs[config].name : nullptr; }
const char* bfp8_fused_config_name(int config) {
  return config_ok(config) ? kConfigs[config].name : nullptr;
}

bfp8_plan bfp8_choose_plan(int M, int N, int K, int num_sms) {
  if (M > 0 && M <= kStreamMaxM) return stream_plan(M, N, K, num_sms);
  if (const TableEntry* t = lookup(kPlanTable, kPlanEntries, M, N, K)) {
    t = balanced_entry(t, M, N, K, num_sms);
    return {t->config, t->splits, 0};
  }
  return heuristic_plan(M, N, K, num_sms, false);
}

// The fused path runs either the quantization kernel followed by the GEMM,
// launched with programmatic dependent launch so the GEMM's prologue and
// first weight loads overlap the quantizer (the unfused GEMM's plan), or a
// GEMM that quantizes its own activations; the fused table says which is
// faster where both were timed, up to its largest M for the shape.
// A quantization-kernel entry always takes the GEMM table's current plan,
// so the fused and unfused routes give the same bits.
bfp8_plan bfp8_choose_fused_plan(int M, int N, int K, int num_sms) {
  if (M > 0 && M <= kStreamMaxM) {
    bfp8_plan plan = stream_plan(M, N, K, num_sms);
    plan.fused = M <= kStreamInGemmMaxM ? BFP8_FUSED_IN_GEMM : BFP8_FUSED_QUANT_KERNEL;
    return plan;
  }
  if (const FusedTableEntry* t = lookup(kFusedPlanTable, kFusedPlanEntries, M, N, K))
    if (t->m >= M && t->mode == BFP8_FUSED_IN_GEMM) return {t->config, t->splits, t->mode};
  bfp8_plan plan = bfp8_choose_plan(M, N, K, num_sms);
  plan.fused = BFP8_FUSED_QUANT_KERNEL;
  return plan;
}

// Quantize-then-GEMM in one call never loses to two separate launches (it
// is the same two kernels, overlapped), so linear always takes it.
int bfp8_prefers_fused(int M, int N, int K) { return M >= 0 && N > 0 && K > 0 ? 1 : 0; }

// The tile configurations only (those with a row-parallel twin).
bfp8_plan bfp8_choose_tp_plan(int M, int N, int K, int num_sms, int fused) {
  if (const TableEntry* t = lookup(kPlanTable, kPlanEntries, M, N, K))
    if (!kConfigs[t->config].stream) {
      t = balanced_entry(t, M, N, K, num_sms);
      if (!kConfigs[t->config].stream) return {t->config, t->splits, fused ? BFP8_FUSED_QUANT_KERNEL : 0};
    }
  return heuristic_plan(M, N, K, num_sms, fused != 0);
}

int bfp8_set_weight_prefetch(int enabled) {
  return g_weight_prefetch.exchange(enabled ? 1 : 0);
}

int bfp8_plan_shape(const bfp8_gemm_problem* p, bfp8_plan plan, int* tiles, int* k_tiles) {
  if (!p || !config_ok(plan.config)) return fail(BFP8_EINVAL, "bad config id");
  const Derived d = derive(*p, plan);
  if (tiles) *tiles = d.tiles;
  if (k_tiles) *k_tiles = d.k_tiles;
  return BFP8_OK;
}

// Weight-streaming configurations hold all tokens in one tile.
int check_tokens(const bfp8_gemm_problem& p, const bfp8_plan& plan) {
  const ConfigEntry& e = kConfigs[plan.config];
  if (e.stream && p.M > e.max_m)
    return fail(BFP8_EINVAL, std::string(e.name) + " handles at most " + std::to_string(e.max_m) + " tokens");
  return BFP8_OK;
}

// CTA-pair configurations have no stream-K schedule.
int check_schedule(const bfp8_plan& plan) {
  if (plan.splits < 0 && kConfigs[plan.config].pair)
    return fail(BFP8_EINVAL, std::string(kConfigs[plan.config].name) + " has no stream-K schedule");
  return BFP8_OK;
}

int64_t bfp8_workspace_bytes(const bfp8_gemm_problem* p, bfp8_plan plan) {
  if (!p || !config_ok(plan.config)) return fail(BFP8_EINVAL, "bad config id");
  if (int r = check_schedule(plan)) return r;
  if (p->M <= 0) return 0;
  if (int r = check_tokens(*p, plan)) return r;
  const bool front = plan.fused && !quantizes_in_kernel(*p, plan);
  return (front ? fused_front_bytes(*p) : 0) + splitk_bytes(*p, plan);
}

int bfp8_counters_needed(const bfp8_gemm_problem* p, bfp8_plan plan) {
  if (!p || !config_ok(plan.config)) return fail(BFP8_EINVAL, "bad config id");
  if (int r = check_schedule(plan)) return r;
  if (p->M <= 0) return 0;
  if (int r = check_tokens(*p, plan)) return r;
  const Derived d = derive(*p, plan);
  return d.splits == 1 ? 0 : d.tiles * (kConfigs[plan.config].bm / 128);
}

int bfp8_launch_quantize(const bfp8_quant_problem* qp, void* stream) {
  if (!qp) return fail(BFP8_EINVAL, "null problem");
  const bfp8_quant_problem& p = *qp;
  if (p.M < 0 || p.K <= 0 || p.K % 8 != 0) return fail(BFP8_EINVAL, "K must be a positive multiple of 8");
  if (p.M == 0) return BFP8_OK;
  if (!p.x || !p.q || !p.s) return fail(BFP8_EINVAL, "null operand pointer");
  if (!aligned16(p.x) || p.ldx < p.K || p.ldx % 8 != 0)
    return fail(BFP8_EINVAL, "x must be row-major with 16-byte aligned rows");
  if ((reinterpret_cast<uintptr_t>(p.q) & 7u) || p.ldq < p.K || p.ldq % 8 != 0)
    return fail(BFP8_EINVAL, "q must be row-major with 8-byte aligned rows");
  if (!(p.eps > 0.f)) return fail(BFP8_EINVAL, "eps must be positive");
  const int sms = current_device_sms(nullptr);
  if (sms <= 0) return cuda_fail(cudaGetLastError(), "cudaGetDevice");
  QuantParams q{static_cast<const __nv_bfloat16*>(p.x), p.ldx, static_cast<uint8_t*>(p.q), p.ldq,
                p.s, p.s_m, p.s_k, p.M, p.K, cdiv(p.K, 128), p.eps};
  return launch_quant(q, static_cast<cudaStream_t>(stream), sms);
}

namespace bfp8 {
namespace {

// Shared checks of the producers' outputs: q (e4m3) and y (bf16) rows.
int check_outputs(const void* q, int64_t ldq, const void* y, int64_t ldy, const float* s, int cols) {
  if (!q && !y) return fail(BFP8_EINVAL, "nothing to write (q and y are both null)");
  if (q && (!s || !aligned16(q) || ldq < cols || ldq % 16 != 0))
    return fail(BFP8_EINVAL, "q must be row-major with 16-byte aligned rows, with scales");
  if (y && (!aligned16(y) || ldy < cols || ldy % 8 != 0))
    return fail(BFP8_EINVAL, "y must be row-major with 16-byte aligned rows");
  return BFP8_OK;
}

int launch_with_pdl(const void* kernel, dim3 grid, void** args, cudaStream_t stream, const char* what) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kProdThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  set_pdl(cfg, attr);
  cudaError_t e = cudaLaunchKernelExC(&cfg, kernel, args);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return BFP8_OK;
}

}  // namespace
}  // namespace bfp8

int bfp8_launch_rmsnorm_quant(const bfp8_rmsnorm_quant_problem* pp, void* stream) {
  if (!pp) return fail(BFP8_EINVAL, "null problem");
  const bfp8_rmsnorm_quant_problem& p = *pp;
  if (p.M < 0 || p.H <= 0 || p.H % 128 != 0 || p.H > kProdChunk * kProdMaxChunks)
    return fail(BFP8_EINVAL, "H must be a positive multiple of 128, at most 16384");
  if (p.M == 0) return BFP8_OK;
  if (!p.x || !p.weight || !aligned16(p.x) || !aligned16(p.weight) || p.ldx < p.H || p.ldx % 8 != 0)
    return fail(BFP8_EINVAL, "x and weight must be 16-byte aligned, x row-major");
  if (p.residual && (!p.residual_out || !aligned16(p.residual) || !aligned16(p.residual_out) || p.ldr < p.H ||
                     p.ldr % 8 != 0 || p.ldro < p.H || p.ldro % 8 != 0))
    return fail(BFP8_EINVAL, "residual and residual_out must be row-major with 16-byte aligned rows");
  if (int r = check_outputs(p.q, p.ldq, p.y, p.ldy, p.s, p.H)) return r;
  if (!(p.eps > 0.f) || !(p.variance_epsilon >= 0.f)) return fail(BFP8_EINVAL, "eps must be positive");
  RmsNormQuantParams k{static_cast<const __nv_bfloat16*>(p.x), p.ldx, static_cast<const __nv_bfloat16*>(p.residual),
                       p.ldr, static_cast<__nv_bfloat16*>(p.residual_out), p.ldro,
                       static_cast<const __nv_bfloat16*>(p.weight), static_cast<__nv_bfloat16*>(p.y), p.ldy,
                       static_cast<uint8_t*>(p.q), p.ldq, p.s, p.s_m, p.s_k, p.M, p.H, p.variance_epsilon, p.eps};
  void* args[] = {&k};
  return launch_with_pdl(reinterpret_cast<const void*>(rmsnorm_quant_kernel), dim3(unsigned(p.M)), args,
                         static_cast<cudaStream_t>(stream), "RMSNorm-quantize launch");
}

int bfp8_launch_silu_mul_quant(const bfp8_silu_mul_quant_problem* pp, void* stream) {
  if (!pp) return fail(BFP8_EINVAL, "null problem");
  const bfp8_silu_mul_quant_problem& p = *pp;
  if (p.M < 0 || p.I <= 0 || p.I % 128 != 0) return fail(BFP8_EINVAL, "I must be a positive multiple of 128");
  if (p.M == 0) return BFP8_OK;
  if (p.M > 65535) return fail(BFP8_EINVAL, "at most 65535 rows per launch");
  if (!p.x || !aligned16(p.x) || p.ldx < 2 * int64_t(p.I) || p.ldx % 8 != 0)
    return fail(BFP8_EINVAL, "x must be row-major [M, 2I] with 16-byte aligned rows");
  if (int r = check_outputs(p.q, p.ldq, p.y, p.ldy, p.s, p.I)) return r;
  if (!(p.eps > 0.f)) return fail(BFP8_EINVAL, "eps must be positive");
  SiluMulQuantParams k{static_cast<const __nv_bfloat16*>(p.x), p.ldx, static_cast<__nv_bfloat16*>(p.y), p.ldy,
                       static_cast<uint8_t*>(p.q), p.ldq, p.s, p.s_m, p.s_k, p.M, p.I, p.eps};
  void* args[] = {&k};
  return launch_with_pdl(reinterpret_cast<const void*>(silu_mul_quant_kernel),
                         dim3(unsigned(cdiv(p.I, kProdChunk)), unsigned(p.M)), args, static_cast<cudaStream_t>(stream),
                         "SiLU-mul-quantize launch");
}

namespace bfp8 {
namespace {

// Checks a row-parallel group against the problem (every pointer the kernel
// will use, this rank's output = p.c).
int check_tp(const bfp8_gemm_problem& p, const bfp8_tp_group& tp) {
  if (tp.world < 1 || tp.world > BFP8_TP_MAX_RANKS) return fail(BFP8_EINVAL, "tp world must be 1..8");
  if (tp.rank < 0 || tp.rank >= tp.world) return fail(BFP8_EINVAL, "tp rank out of range");
  for (int q = 0; q < tp.world; ++q) {
    if (!tp.partials[q] || !tp.counters[q] || !tp.out[q]) return fail(BFP8_EINVAL, "null tp buffer");
    if (!aligned16(tp.partials[q]) || !aligned16(tp.out[q]) || (reinterpret_cast<uintptr_t>(tp.counters[q]) & 7u))
      return fail(BFP8_EINVAL, "tp buffers must be 16-byte aligned (counters 8-byte)");
  }
  if (tp.out[tp.rank] != p.c) return fail(BFP8_EINVAL, "c must be this rank's tp output (out[rank])");
  return BFP8_OK;
}

// Shared-memory layout of a weight-streaming launch: the ring of stages
// (`group` K blocks each: weight tiles, e4m3 activation tiles and, when the
// kernel quantizes, bf16 activation tiles), then the per-position token and
// weight scales and the barriers.  Preferred: at most 112 KB, so that two
// CTAs fit on an SM (the next call's CTAs start beside this call's); stages
// of 2 K blocks x 3 when they fit, else smaller.  Problems whose scale
// arrays do not allow that use the whole of shared memory.
struct StreamLayout {
  int stages, group, smem;
  uint32_t stage_bytes, off_sa, off_sb, off_bars;
};

constexpr int kStreamPairSmem = 112 * 1024;
constexpr int64_t kStreamDeepRingSpan = 16;  // K blocks per CTA from which the deep ring wins

int stream_layout(int bn, bool quant, int M, const Derived& d, StreamLayout* out) {
  const int64_t span = (d.sk_work + d.sk_grid - 1) / d.sk_grid;
  const int acc = 256 / bn;  // StreamCfg::ACC_BUFS
  auto a16 = [](int64_t x) { return (x + 15) & ~int64_t(15); };
  auto fits = [&](int s, int group, int limit, StreamLayout* o) {
    // (1024-byte multiples: every stage's tiles keep the 128-byte swizzle's alignment)
    const int64_t stage = (int64_t(group) * (16384 + bn * 128 + (quant ? std::min(M, bn) * 256 : 0)) + 1023) & ~int64_t(1023);
    const int64_t off_sa = int64_t(s) * stage;
    const int64_t off_sb = off_sa + a16(span * bn * 4);
    const int64_t off_bars = off_sb + a16(span * 4);
    const int64_t end = off_bars + (4 * s + 2 * acc + 1) * 8 + 16;
    if (1024 + end > limit) return false;
    *o = {s, group, int(1024 + end), uint32_t(stage), uint32_t(off_sa), uint32_t(off_sb), uint32_t(off_bars)};
    return true;
  };
  // A CTA whose range is long (many more K blocks than a 112 KB ring holds)
  // streams for most of the call: it gains more from a deep ring of its own
  // than from a second CTA of the next call beside it.
  if (span < kStreamDeepRingSpan) {
    const int pair[][2] = {{3, 2}, {2, 2}, {3, 1}, {2, 1}};  // {stages, K blocks per stage}, two CTAs per SM
    for (const auto& t : pair)
      if (fits(t[0], t[1], kStreamPairSmem, out)) return BFP8_OK;
  }
  const int alone[][2] = {{3, 4}, {2, 4}, {4, 2}, {3, 2}, {2, 2}, {3, 1}, {2, 1}};
  for (const auto& t : alone)
    if (fits(t[0], t[1], kMaxSmem, out)) return BFP8_OK;
  return fail(BFP8_EINVAL, "this problem's per-CTA scale arrays do not fit a weight-streaming configuration's "
                           "shared memory (use more CTAs or another configuration)");
}

int launch_stream(const bfp8_gemm_problem& p, const void* x_bf16, const bfp8_plan& plan, const Derived& d,
                  bool in_kernel, uint8_t* ws, int* counters, int dev, cudaStream_t stream) {
  const ConfigEntry& e = kConfigs[plan.config];
  if (d.sk_work >= (int64_t(1) << 31)) return fail(BFP8_EINVAL, "too many weight tiles x K blocks for " + std::string(e.name));
  StreamLayout lay;
  if (int r = stream_layout(e.bn, in_kernel, p.M, d, &lay)) return r;
  StreamParams sp;
  std::memset(&sp, 0, sizeof(sp));
  if (int r = make_map(&sp.map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.b, uint64_t(p.K), uint64_t(p.N),
                       uint64_t(p.ldb), 128, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return r;
  if (in_kernel) {
    // bf16 activations: [BN rows x 128 values] boxes, quantized in the kernel
    const int rows = std::min(p.M, e.bn);
    if (int r = make_map(&sp.map_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x_bf16, uint64_t(p.K), uint64_t(p.M),
                         uint64_t(p.lda) * 2, 128, uint32_t(rows), CU_TENSOR_MAP_SWIZZLE_NONE))
      return r;
    sp.eps = p.eps;
    sp.x_bytes = uint32_t(rows) * 256u;
  } else {
    if (int r = make_map(&sp.map_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.a, uint64_t(p.K), uint64_t(p.M),
                         uint64_t(p.lda), 128, uint32_t(e.bn), CU_TENSOR_MAP_SWIZZLE_128B))
      return r;
    sp.sa = p.sa;
    sp.sa_m = p.sa_m;
    sp.sa_k = p.sa_k;
  }
  sp.sb = p.sb;
  sp.sb_n = p.sb_n;
  sp.sb_k = p.sb_k;
  sp.c = static_cast<__nv_bfloat16*>(p.c);
  sp.ldc = p.ldc;
  sp.workspace = reinterpret_cast<float*>(ws);
  sp.counters = counters;
  sp.M = p.M;
  sp.N = p.N;
  sp.K = p.K;
  sp.tiles = d.tiles;
  sp.k_tiles = d.k_tiles;
  sp.max_pieces = d.splits;
  sp.work = int(d.sk_work);
  sp.work_q = int(d.sk_work / d.sk_grid);
  sp.work_r = int(d.sk_work % d.sk_grid);
  sp.stages = lay.stages;
  sp.group = lay.group;
  sp.early = g_weight_prefetch.load(std::memory_order_relaxed) ? lay.stages : 0;
  sp.stage_bytes = lay.stage_bytes;
  sp.off_sa = lay.off_sa;
  sp.off_sb = lay.off_sb;
  sp.off_bars = lay.off_bars;
  if (int r = ensure_smem_attr(plan.config, dev, in_kernel)) return r;
  (in_kernel ? e.launch_stream_q : e.launch_stream)(sp, d.sk_grid, lay.smem, true, stream);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(err, "weight-streaming GEMM launch");
  return BFP8_OK;
}

int launch_gemm_impl(const bfp8_gemm_problem* pp, bfp8_plan plan, float* workspace, int* counters,
                     const bfp8_tp_group* tp, void* stream_) {
  if (!pp) return fail(BFP8_EINVAL, "null problem");
  if (!config_ok(plan.config)) return fail(BFP8_EINVAL, "config out of range");
  if (plan.splits == 0) return fail(BFP8_EINVAL, "splits must be >= 1 (or negative: stream-K)");
  if (int r = check_schedule(plan)) return r;
  bfp8_gemm_problem p = *pp;
  const bool fused = plan.fused != 0;
  if (int r = check_problem(p, fused)) return r;
  if (p.M == 0) return BFP8_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int dev = 0;
  const int sms = current_device_sms(&dev);
  if (sms <= 0) return cuda_fail(cudaGetLastError(), "cudaGetDevice");

  const Derived d = derive(p, plan);
  const bool in_kernel = quantizes_in_kernel(p, plan);
  if (int r = check_tokens(p, plan)) return r;
  if (tp && kConfigs[plan.config].stream)
    return fail(BFP8_EINVAL, std::string(kConfigs[plan.config].name) + " has no row-parallel variant");
  if (((fused && !in_kernel) || d.splits > 1) && !workspace) return fail(BFP8_EINVAL, "workspace required");
  if (d.splits > 1 && !counters) return fail(BFP8_EINVAL, "split-K counters required");

  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  const void* x_bf16 = p.a;
  if (fused && !in_kernel) {
    // gemm_bf16: quantize x into the front of the workspace (M-major
    // scales), then the GEMM reads it like any quantized input.
    uint8_t* q = ws;
    float* s = reinterpret_cast<float*>(ws + align256(int64_t(p.M) * p.K));
    QuantParams qp{static_cast<const __nv_bfloat16*>(p.a), p.lda, q, p.K, s, 1, p.M, p.M, p.K,
                   cdiv(p.K, 128), p.eps};
    if (int r = launch_quant(qp, stream, sms)) return r;
    p.a = q;
    p.lda = p.K;
    p.sa = s;
    p.sa_m = 1;
    p.sa_k = p.M;
    ws += fused_front_bytes(*pp);
  }

  const ConfigEntry& e = kConfigs[plan.config];
  if (e.stream) return launch_stream(p, x_bf16, plan, d, in_kernel, ws, counters, dev, stream);
  GemmParams gp;
  std::memset(&gp, 0, sizeof(gp));
  if (in_kernel) {
    // The kernel reads the bf16 activations and quantizes them itself;
    // operand B's tensor map is not used.
    gp.x = static_cast<const __nv_bfloat16*>(x_bf16);
    gp.ldx = p.lda;
    gp.eps = p.eps;
  }
  // Operand tiles: 128 rows of the MMA A operand, BN rows of the B operand
  // (a CTA pair: each CTA loads BN / 4 rows of each of the two column
  // blocks), one 128-byte K block each, 128-byte swizzle.  Activations are A
  // in the normal order and B in the swapped one.
  const void* a_src = e.swap ? p.b : p.a;
  const void* b_src = in_kernel ? p.b : (e.swap ? p.a : p.b);  // in-kernel: placeholder, unused
  const int64_t a_ld = e.swap ? p.ldb : p.lda, b_ld = (e.swap && !in_kernel) ? p.lda : p.ldb;
  const int a_rows = e.swap ? p.N : p.M, b_rows = in_kernel ? p.N : (e.swap ? p.M : p.N);
  if (int r = make_map(&gp.map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, a_src, uint64_t(p.K),
                       uint64_t(a_rows), uint64_t(a_ld), 128, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return r;
  if (int r = make_map(&gp.map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, b_src, uint64_t(p.K),
                       uint64_t(b_rows), uint64_t(b_ld), 128, uint32_t(e.pair ? e.bn / 4 : e.bn),
                       CU_TENSOR_MAP_SWIZZLE_128B))
    return r;
  // Output: normal order stores [32 rows x 32 columns] chunks (64-byte
  // swizzle); swapped order stores [BN tokens x 32 columns] tiles.
  if (int r = e.swap ? make_map(&gp.map_c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.c, uint64_t(p.N),
                                uint64_t(p.M), uint64_t(p.ldc) * 2, 32, uint32_t(e.bn),
                                CU_TENSOR_MAP_SWIZZLE_NONE)
                     : make_map(&gp.map_c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.c, uint64_t(p.N),
                                uint64_t(p.M), uint64_t(p.ldc) * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    return r;
  gp.sa = p.sa;
  gp.sa_m = p.sa_m;
  gp.sa_k = p.sa_k;
  gp.sb = p.sb;
  gp.sb_n = p.sb_n;
  gp.sb_k = p.sb_k;
  gp.workspace = reinterpret_cast<float*>(ws);
  gp.counters = counters;
  gp.M = p.M;
  gp.N = p.N;
  gp.K = p.K;
  gp.tiles_r = d.tiles_r;
  gp.tiles_c = d.tiles_c;
  gp.tiles = d.tiles;
  gp.k_tiles = d.k_tiles;
  gp.k_per_split = d.k_per_split;
  gp.splits = d.splits;
  gp.units = d.sk_grid > 0 ? int(d.sk_work) : d.tiles * d.splits;
  gp.sk_grid = d.sk_grid;
  gp.sk_work = d.sk_work;
  // Raster: when all row tiles of the MMA A operand fit comfortably in L2,
  // sweep them all for each column tile, so A stays resident and B streams
  // from HBM once; otherwise groups of 8 row tiles (the reference's
  // group_m).  Swapped order: A is the weights, B the few token rows.
  const int64_t a_bytes = int64_t(d.tiles_r) * e.bm * p.K;
  gp.group_r = e.swap || a_bytes <= (int64_t(48) << 20) ? d.tiles_r : 1024 / e.bm;
  gp.stream_b = (e.swap || p.M <= 128) ? 1 : 0;  // weights read once: evict them first
  gp.pdl = g_weight_prefetch.load(std::memory_order_relaxed) ? 1 : 0;  // early weight tiles
  if (tp) {
    gp.tp_world = tp->world;
    gp.tp_rank = tp->rank;
    gp.tp_wait = tp->wait ? 1 : 0;
    // Rank r starts at the first tile of rank r + 1's block (tile t belongs
    // to rank floor(t * world / tiles), so block q starts at
    // ceil(q * tiles / world)) and reaches its own block last.
    const int64_t next = (tp->rank + 1) % tp->world;
    gp.tp_rot = int((next * d.tiles + tp->world - 1) / tp->world) % d.tiles;
    for (int q = 0; q < tp->world; ++q) {
      gp.tp_partials[q] = tp->partials[q];
      gp.tp_counters[q] = tp->counters[q];
      gp.tp_out[q] = static_cast<__nv_bfloat16*>(tp->out[q]);
    }
    gp.tp_ldo = p.ldc;
  }

  if (int r = ensure_smem_attr(plan.config, dev, in_kernel, tp != nullptr)) return r;
  // One CTA (a pair: two) per SM, persistent over the units.
  const int grid = d.sk_grid > 0 ? d.sk_grid : e.pair ? 2 * std::min(gp.units, sms / 2) : std::min(gp.units, sms);
  (in_kernel ? (tp ? e.launch_fused_tp : e.launch_fused) : (tp ? e.launch_tp : e.launch))(gp, grid, stream);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(err, "GEMM kernel launch");
  return BFP8_OK;
}

}  // namespace
}  // namespace bfp8

int bfp8_launch_gemm(const bfp8_gemm_problem* p, bfp8_plan plan, float* workspace, int* counters, void* stream) {
  return launch_gemm_impl(p, plan, workspace, counters, nullptr, stream);
}

int bfp8_tp_tiles(const bfp8_gemm_problem* p, bfp8_plan plan) {
  if (!p || !config_ok(plan.config)) return fail(BFP8_EINVAL, "bad config id");
  if (kConfigs[plan.config].stream)
    return fail(BFP8_EINVAL, std::string(kConfigs[plan.config].name) + " has no row-parallel variant");
  if (int r = check_schedule(plan)) return r;
  if (p->M <= 0) return 0;
  const Derived d = derive(*p, plan);
  return d.tiles * (kConfigs[plan.config].bm / 128);
}

int64_t bfp8_tp_partial_bytes(const bfp8_gemm_problem* p, bfp8_plan plan, int world) {
  if (world < 1 || world > BFP8_TP_MAX_RANKS) return fail(BFP8_EINVAL, "tp world must be 1..8");
  const int tiles = bfp8_tp_tiles(p, plan);
  if (tiles < 0) return tiles;
  return int64_t(world) * tiles * 128 * kConfigs[plan.config].bn * int64_t(sizeof(float));
}

int bfp8_launch_gemm_tp(const bfp8_gemm_problem* p, bfp8_plan plan, float* workspace, int* counters,
                        const bfp8_tp_group* tp, void* stream) {
  if (!p || !tp) return fail(BFP8_EINVAL, "null problem or tp group");
  if (!config_ok(plan.config)) return fail(BFP8_EINVAL, "config out of range");
  if (p->M > 0)
    if (int r = check_tp(*p, *tp)) return r;
  return launch_gemm_impl(p, plan, workspace, counters, tp, stream);
}

static_assert(sizeof(cudaIpcMemHandle_t) == BFP8_IPC_HANDLE_BYTES, "CUDA IPC handle size");

int bfp8_tp_alloc(int64_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes <= 0) return fail(BFP8_EINVAL, "tp alloc: null output or non-positive size");
  *ptr = nullptr;
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, size_t(bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(tp buffer)");
  e = cudaMemset(d, 0, size_t(bytes));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, d);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "tp buffer set-up");
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = d;
  return BFP8_OK;
}

int bfp8_tp_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(BFP8_EINVAL, "tp open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return BFP8_OK;
}

int bfp8_tp_close(void* ptr) {
  if (!ptr) return BFP8_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? BFP8_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int bfp8_tp_free(void* ptr) {
  if (!ptr) return BFP8_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? BFP8_OK : cuda_fail(e, "cudaFree(tp buffer)");
}

int bfp8_launch_gemm_noalloc(const bfp8_gemm_problem* p, bfp8_plan plan, void* stream) {
  if (!p) return fail(BFP8_EINVAL, "null problem");
  if (!config_ok(plan.config)) return fail(BFP8_EINVAL, "config out of range");
  if (plan.splits == 0) return fail(BFP8_EINVAL, "splits must be >= 1 (or negative: stream-K)");
  if (p->M <= 0) return bfp8_launch_gemm(p, plan, nullptr, nullptr, stream);
  const int64_t ws = bfp8_workspace_bytes(p, plan);
  const int counters = bfp8_counters_needed(p, plan);
  if (ws < 0 || counters < 0) return int(ws < 0 ? ws : counters);
  const int64_t ws_room = int64_t(BFP8_STATIC_SCRATCH_BYTES) - BFP8_STATIC_COUNTER_BYTES;
  if (ws > ws_room || int64_t(counters) * 4 > BFP8_STATIC_COUNTER_BYTES)
    return fail(BFP8_EINVAL, "this plan needs " + std::to_string(ws) + " bytes of workspace and " +
                                 std::to_string(counters) + " counters; the fixed scratch holds " +
                                 std::to_string(ws_room) + " bytes and " +
                                 std::to_string(BFP8_STATIC_COUNTER_BYTES / 4) +
                                 " counters (use fewer splits, or bfp8_launch_gemm with a workspace)");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  unsigned char* base = nullptr;
  if (int r = static_scratch(dev, &base)) return r;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The kernels leave every counter they use at zero, so after a normal call
  // this clear changes nothing; it is here for the call after one whose
  // bounded wait gave up (its counters were left mid-count), since the
  // array outlives every call.  One small memset on the stream per split-K
  // call, kept for that robustness.
  if (counters > 0) {
    e = cudaMemsetAsync(base, 0, size_t(counters) * 4, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(static scratch counters)");
  }
  return bfp8_launch_gemm(p, plan, ws ? reinterpret_cast<float*>(base + BFP8_STATIC_COUNTER_BYTES) : nullptr,
                          counters ? reinterpret_cast<int*>(base) : nullptr, stream);
}

int64_t bfp8_device_status(int reset) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  unsigned long long v = 0;
  e = cudaMemcpyFromSymbol(&v, bfp8::g_status, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(status)");
  if (reset && v) {
    const unsigned long long zero = 0;
    e = cudaMemcpyToSymbol(bfp8::g_status, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(status)");
  }
  return int64_t(v & 0x7fffffffffffffffull);
}

}  // extern "C"

// ---- roofline probes (no reference counterpart) ------------------------------------

namespace {

template <int N>
int run_probe_mma(int iters, double* tflops, double* macs_per_clock) {
  using namespace bfp8;
  const int sms = current_device_sms(nullptr);
  if (sms <= 0) return cuda_fail(cudaGetLastError(), "cudaGetDevice");
  constexpr int kSmem = 150 * 1024;  // one CTA per SM
  cudaError_t err = cudaFuncSetAttribute(probe_mma_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (err != cudaSuccess) return cuda_fail(err, "cudaFuncSetAttribute (probe)");
  unsigned long long* clocks = nullptr;
  if ((err = cudaMalloc(&clocks, sizeof(unsigned long long) * sms)) != cudaSuccess)
    return cuda_fail(err, "cudaMalloc (probe)");
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  probe_mma_kernel<N><<<sms, 128, kSmem>>>(8, clocks);  // warm-up
  cudaEventRecord(e0);
  probe_mma_kernel<N><<<sms, 128, kSmem>>>(iters, clocks);
  cudaEventRecord(e1);
  err = cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  std::vector<unsigned long long> h(sms);
  if (err == cudaSuccess) err = cudaMemcpy(h.data(), clocks, sizeof(unsigned long long) * sms, cudaMemcpyDeviceToHost);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(clocks);
  if (err != cudaSuccess) return cuda_fail(err, "probe launch");
  std::sort(h.begin(), h.end());
  const double macs = double(iters) * 4 * 128 * N * 32;  // per CTA
  if (tflops) *tflops = 2.0 * macs * sms / (double(ms) * 1e-3) / 1e12;
  if (macs_per_clock) *macs_per_clock = macs / double(h[h.size() / 2]);
  return BFP8_OK;
}

}  // namespace

extern "C" int bfp8_probe_mma(int n, int iters, double* tflops, double* macs_per_clock) {
  if (iters <= 0) return fail(BFP8_EINVAL, "iters must be positive");
  if (n == 256) return run_probe_mma<256>(iters, tflops, macs_per_clock);
  if (n == 128) return run_probe_mma<128>(iters, tflops, macs_per_clock);
  return fail(BFP8_EINVAL, "probe n must be 128 or 256");
}

extern "C" int bfp8_probe_hbm_read(const void* buf, int64_t bytes, int reps, double* gbs) {
  if (!buf || bytes < 16 || reps <= 0 || !aligned16(buf)) return fail(BFP8_EINVAL, "probe buffer");
  const int sms = current_device_sms(nullptr);
  if (sms <= 0) return cuda_fail(cudaGetLastError(), "cudaGetDevice");
  const int grid = sms * 8;
  uint32_t* sink = nullptr;
  cudaError_t err = cudaMalloc(&sink, sizeof(uint32_t) * grid * 256);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMalloc (probe)");
  const int64_t words = bytes / 16;
  const uint4* p = static_cast<const uint4*>(buf);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  bfp8::probe_read_kernel<<<grid, 256>>>(p, words, sink);  // warm-up
  cudaEventRecord(e0);
  for (int r = 0; r < reps; ++r) bfp8::probe_read_kernel<<<grid, 256>>>(p, words, sink);
  cudaEventRecord(e1);
  err = cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(sink);
  if (err != cudaSuccess) return cuda_fail(err, "probe launch");
  if (gbs) *gbs = double(words) * 16 * reps / (double(ms) * 1e-3) / 1e9;
  return BFP8_OK;
}

extern "C" int bfp8_probe_block(const void* a, const void* b, float* d, void* stream) {
  if (!a || !b || !d || !aligned16(a) || !aligned16(b)) return fail(BFP8_EINVAL, "probe operands");
  constexpr int kSmem = 1024 + 128 * 128 + 32 * 128;
  cudaError_t err = cudaFuncSetAttribute(bfp8::probe_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (err != cudaSuccess) return cuda_fail(err, "cudaFuncSetAttribute (probe)");
  bfp8::probe_block_kernel<<<1, 128, kSmem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(a), static_cast<const uint8_t*>(b), d);
  err = cudaGetLastError();
  return err == cudaSuccess ? BFP8_OK : cuda_fail(err, "probe launch");
}

extern "C" int bfp8_probe_quantizer(float eps, unsigned long long* mismatches, unsigned long long* first) {
  if (!mismatches || !(eps > 0.f)) return bfp8::fail(BFP8_EINVAL, "probe arguments");
  unsigned long long* d = nullptr;
  cudaError_t err = cudaMalloc(&d, 2 * sizeof(unsigned long long));
  if (err != cudaSuccess) return bfp8::cuda_fail(err, "cudaMalloc (probe)");
  err = cudaMemset(d, 0, 2 * sizeof(unsigned long long));
  if (err == cudaSuccess) {
    bfp8::probe_quant_kernel<<<0x7F80, 256>>>(eps, d);
    err = cudaGetLastError();
  }
  unsigned long long h[2] = {0, 0};
  if (err == cudaSuccess) err = cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (err != cudaSuccess) return bfp8::cuda_fail(err, "probe launch");
  *mismatches = h[0];
  if (first) *first = h[1];
  return BFP8_OK;
}

extern "C" int bfp8_probe_scale(unsigned long long* mismatches, unsigned long long* first) {
  if (!mismatches) return bfp8::fail(BFP8_EINVAL, "probe arguments");
  unsigned long long* d = nullptr;
  cudaError_t err = cudaMalloc(&d, 2 * sizeof(unsigned long long));
  if (err != cudaSuccess) return bfp8::cuda_fail(err, "cudaMalloc (probe)");
  err = cudaMemset(d, 0, 2 * sizeof(unsigned long long));
  if (err == cudaSuccess) {
    bfp8::probe_scale_kernel<<<148 * 16, 256>>>(d);
    err = cudaGetLastError();
  }
  unsigned long long h[2] = {0, 0};
  if (err == cudaSuccess) err = cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (err != cudaSuccess) return bfp8::cuda_fail(err, "probe launch");
  *mismatches = h[0];
  if (first) *first = h[1];
  return BFP8_OK;
}
