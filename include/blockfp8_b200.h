/*
 * blockfp8_b200 -- C ABI of the B200 (sm_100a) block-FP8 linear hot path.
 *
 *   C[M, N] (bf16) = sum_kb sa[m, kb] * sb[n / 128, kb] * sum_{k in kb} A[m, k] * B[n, k]
 *
 * A [M, K] and B [N, K] are float8_e4m3fn codes, K-contiguous ("TN"); sa is
 * float32 [M, ceil(K/128)] with any strides; sb is float32
 * [ceil(N/128), ceil(K/128)]; C is bf16 [M, N].  All strides are in elements.
 *
 * This header is the drop-in replacement for the reference's host interface
 * (simon-jd/blockfp8 csrc/blockfp8.h:17-76, a C++ namespace API used only by
 * csrc/ops.cpp).  Each declaration names the reference function it replaces.
 * Differences: plain C (extern "C"), structs passed by pointer, errors are
 * returned as negative status codes with the message in bfp8_last_error()
 * instead of a thrown std::runtime_error, and the CUDA stream is passed as
 * void* (a cudaStream_t), so the header needs no CUDA include.
 *
 * Every pointer in a problem struct is a device pointer on the current CUDA
 * device.  Launch functions are asynchronous on the given stream.
 */
#ifndef BLOCKFP8_B200_H
#define BLOCKFP8_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BFP8_OK 0
#define BFP8_EINVAL (-1)  /* bad argument: shape, alignment, config id, ... */
#define BFP8_ECUDA (-2)   /* a CUDA runtime or driver call failed */

/* Problem descriptor; replaces blockfp8::GemmProblem (csrc/blockfp8.h:17-30).
 * With a fused plan, a points at bf16 activations [M, K] (row stride lda),
 * which are quantized per row per 128-wide K group with the amax floored at
 * eps; sa is then unused. */
typedef struct bfp8_gemm_problem {
  const void* a;
  int64_t lda;
  const void* b;
  int64_t ldb;
  const float* sa;
  int64_t sa_m, sa_k;
  const float* sb;
  int64_t sb_n, sb_k;
  void* c;
  int64_t ldc;
  int M, N, K;
  float eps;
} bfp8_gemm_problem;

/* Kernel choice; replaces blockfp8::Plan (csrc/blockfp8.h:32-36). */
typedef struct bfp8_plan {
  int config; /* index into the compiled (fused, if fused) configurations */
  int splits; /* K splits (1 = no split-K); negative: stream-K, -splits CTAs
                 share all tiles' K blocks evenly, each tile's parts summed
                 in K order (deterministic) */
  int fused;  /* 0: A is e4m3 with scales sa; nonzero: A is bf16 and is
                 quantized as part of the call, by a quantization kernel
                 into the workspace ahead of the GEMM (BFP8_FUSED_QUANT_KERNEL)
                 or, for BFP8_FUSED_IN_GEMM, inside the GEMM kernel itself
                 where the configuration has that variant and one split's K
                 range fits its resident operand (else as QUANT_KERNEL).
                 Results are bit-identical either way. */
} bfp8_plan;

#define BFP8_FUSED_QUANT_KERNEL 1
#define BFP8_FUSED_IN_GEMM 2

/* Activation quantization problem; replaces blockfp8::QuantProblem
 * (csrc/blockfp8.h:66-75): x [M, K] bf16 (row stride ldx) -> q [M, K] e4m3
 * (row stride ldq) and one float scale per row per 128-wide K group at
 * s[m * s_m + kb * s_k].  K must be a multiple of 8. */
typedef struct bfp8_quant_problem {
  const void* x;
  int64_t ldx;
  void* q;
  int64_t ldq;
  float* s;
  int64_t s_m, s_k;
  int M, K;
  float eps;
} bfp8_quant_problem;

/* Configuration tables; replace num_configs / config_name / num_fused_configs
 * / fused_config_name (csrc/blockfp8.h:38-41).  Names are static strings. */
int bfp8_num_configs(void);
const char* bfp8_config_name(int config);
int bfp8_num_fused_configs(void);
const char* bfp8_fused_config_name(int config);

/* The built-in plan; replace choose_plan / choose_fused_plan
 * (csrc/blockfp8.h:43-45).  num_sms = the device's multiprocessor count. */
bfp8_plan bfp8_choose_plan(int M, int N, int K, int num_sms);
bfp8_plan bfp8_choose_fused_plan(int M, int N, int K, int num_sms);
/* (choose_fused_plan's plan.fused is the faster of the two fused modes for
 * the shape, as tuned on a B200.) */

/* The built-in plan among the configurations that have a row-parallel twin
 * (bfp8_launch_gemm_tp); fused != 0 asks for BFP8_FUSED_QUANT_KERNEL.  The
 * weight-streaming configurations ("w128d...") that bfp8_choose_plan picks
 * for decode batches have none.  No counterpart in the reference. */
bfp8_plan bfp8_choose_tp_plan(int M, int N, int K, int num_sms, int fused);

/* Whether linear runs this shape through the fused path; replaces
 * prefers_fused (csrc/blockfp8.h:47-50).  Returns 0 or 1. */
int bfp8_prefers_fused(int M, int N, int K);

/* Tiles and K tiles of a plan; replaces plan_shape (csrc/blockfp8.h:52-53).
 * Returns BFP8_OK or BFP8_EINVAL (bad config id). */
int bfp8_plan_shape(const bfp8_gemm_problem* p, bfp8_plan plan, int* tiles, int* k_tiles);

/* Scratch of one launch: fp32 split-K partial tiles, preceded for a fused
 * plan by the quantized activations and their scales (bytes); and the int
 * split-K arrival counters.  Replace workspace_bytes / counters_needed
 * (csrc/blockfp8.h:55-57).  Workspace is 0 for an unfused one-split plan,
 * counters 0 for any one-split plan.  Negative on a bad config id. */
int64_t bfp8_workspace_bytes(const bfp8_gemm_problem* p, bfp8_plan plan);
int bfp8_counters_needed(const bfp8_gemm_problem* p, bfp8_plan plan);

/* Launch the GEMM; replaces launch_gemm (csrc/blockfp8.h:59-61).
 * workspace: bfp8_workspace_bytes() bytes (may be NULL when that is 0).
 * counters: bfp8_counters_needed() ints that are zero on entry; the kernel
 * leaves them zero.  Calls that overlap on the GPU must not share counters
 * or workspace.  A fused plan quantizes p->a (bf16) into the front of the
 * workspace first.  Returns BFP8_OK, BFP8_EINVAL or BFP8_ECUDA. */
int bfp8_launch_gemm(const bfp8_gemm_problem* p, bfp8_plan plan, float* workspace, int* counters,
                     void* stream);

/* The same launch without any caller-provided or allocated device memory.
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory on this path -- a serving loop whose device memory is all reserved
 * up front, a host runtime bound through FFI without a CUDA allocator, code
 * that must not risk cudaMalloc's implicit device synchronisation -- the
 * split-K partials, the split-K counters and the fused path's quantized
 * activations live in one fixed array in the library's device memory,
 * BFP8_STATIC_SCRATCH_BYTES per device, held by every GPU that loads the
 * library until the process exits.  A plan that needs more than it holds
 * (bfp8_workspace_bytes() above BFP8_STATIC_SCRATCH_BYTES -
 * BFP8_STATIC_COUNTER_BYTES, or more than BFP8_STATIC_COUNTER_BYTES / 4
 * counters) is rejected with BFP8_EINVAL and nothing is launched.  The first
 * call on a device looks the array's address up (cudaGetSymbolAddress), so
 * make it before any stream capture.  Each call clears the counters it uses
 * (cudaMemsetAsync on the stream; the kernels leave them zero, so this only
 * matters after a call whose bounded wait gave up); every call shares the
 * one array, so calls
 * that overlap on the GPU (other streams, other host threads) race and must
 * be serialised by the caller.  Allocates nothing.  Same results as
 * bfp8_launch_gemm under the same plan. */
#define BFP8_STATIC_SCRATCH_BYTES (16u << 20)
#define BFP8_STATIC_COUNTER_BYTES (64u << 10)
int bfp8_launch_gemm_noalloc(const bfp8_gemm_problem* p, bfp8_plan plan, void* stream);

/* ---- row-parallel linear with its all-reduce inside the GEMM ------------------
 * Replaces the GEMM + NCCL all-reduce of a row-parallel (K-split) layer --
 * the o and down projections of a tensor-parallel model, where vLLM's
 * RowParallelLinear calls the block-FP8 GEMM (blockfp8_vllm/kernel.py:42-61)
 * and then all-reduces the bf16 outputs.  Every rank of a group of `world`
 * GPUs launches the same problem shape and plan over its own K slice.
 * Tiles belong to ranks in contiguous blocks and each rank's schedule
 * reaches its own block last.  A tile's fp32 sum goes to its owner's
 * partial buffer (over NVLink for the other ranks); the arrival that
 * completes the tile's count -- usually the owner's own -- sums the `world`
 * partials in rank order from zero, rounds once to bf16 and stores the tile
 * into every rank's output; so the result is the same on every rank and
 * from call to call.  No CTA waits for another rank inside the tile loop;
 * with wait = 1 one thread waits (bounded, about 2 s, then the device
 * status records site 8) at the end until this rank's output is complete.
 *
 * Buffers, per rank, mapped into every other rank (bfp8_tp_alloc /
 * bfp8_tp_open):
 *   partials: bfp8_tp_partial_bytes() (with this world size) bytes;
 *   counters: 2 + bfp8_tp_tiles() unsigned 64-bit, zero at allocation:
 *             [0] tiles delivered to this rank, [1] tiles this rank has
 *             taken (both grow by bfp8_tp_tiles() per call), [2 + t]
 *             arrivals on tile t (the kernel resets them);
 *   out:      the bf16 output [M, N] (row stride p->ldc, the same on every
 *             rank); p->c must be out[rank].
 * The host keeps no per-call state, so a sequence of calls can be captured
 * and replayed.  All ranks make the same calls in the same order; a call's
 * output stays valid until the group's next call.  After an error (a
 * bounded wait gave up) the counters are no longer consistent: make a new
 * group.  wait = 0 leaves the ordering to the caller (e.g. ranks emulated
 * one after another on one GPU).  No counterpart in the reference. */
#define BFP8_TP_MAX_RANKS 8
typedef struct bfp8_tp_group {
  int world, rank;
  int wait;
  float* partials[BFP8_TP_MAX_RANKS];
  unsigned long long* counters[BFP8_TP_MAX_RANKS];
  void* out[BFP8_TP_MAX_RANKS];
} bfp8_tp_group;

int bfp8_tp_tiles(const bfp8_gemm_problem* p, bfp8_plan plan);
int64_t bfp8_tp_partial_bytes(const bfp8_gemm_problem* p, bfp8_plan plan, int world);
int bfp8_launch_gemm_tp(const bfp8_gemm_problem* p, bfp8_plan plan, float* workspace, int* counters,
                        const bfp8_tp_group* tp, void* stream);

/* Peer buffers for a group: bfp8_tp_alloc cudaMallocs `bytes` (zeroed) on
 * the current device and writes its CUDA IPC handle (64 bytes) to `handle`;
 * another rank's process maps it with bfp8_tp_open (peer access enabled on
 * first use) and unmaps it with bfp8_tp_close; the owner frees it with
 * bfp8_tp_free.  No counterpart in the reference. */
#define BFP8_IPC_HANDLE_BYTES 64
int bfp8_tp_alloc(int64_t bytes, void** ptr, void* handle);
int bfp8_tp_open(const void* handle, void** ptr);
int bfp8_tp_close(void* ptr);
int bfp8_tp_free(void* ptr);

/* Programmatic dependent launch.  Every GEMM and quantizer launch may start
 * while the previous kernel of its stream is still running: it waits
 * (griddepcontrol.wait) before reading activations or activation scales and
 * before writing anything, and it lets the next kernel start early.  With
 * weight prefetch on (the default) the GEMMs also request their first weight
 * tiles and read weight scales before that wait, so that behind another
 * GEMM the weight stream never stops.  Weights and weight scales must
 * therefore not be written by the kernel that immediately precedes the call
 * in its stream (model weights are written once, long before).  Turn it off
 * for code that writes weights right before using them.  Process-wide;
 * returns the previous setting.  No counterpart in the reference. */
int bfp8_set_weight_prefetch(int enabled);

/* Launch the activation quantizer; replaces launch_quantize
 * (csrc/blockfp8.h:76).  Returns BFP8_OK, BFP8_EINVAL or BFP8_ECUDA. */
int bfp8_launch_quantize(const bfp8_quant_problem* p, void* stream);

/* The layers that feed a block-FP8 linear, emitting its e4m3 operand and
 * M-major scales in the same kernel (no quantization launch between them and
 * the GEMM).  No reference counterpart: the reference quantizes activations
 * in a separate kernel (csrc/quant_sm89.cu) and notes fusing into the
 * previous layer as outside its kernels (docs/design-tradeoffs.md:158-160).
 * Codes and scales equal bfp8_launch_quantize applied to the bf16 output y,
 * which the kernels also write when y is not null; q null = y only.
 *
 * RMSNorm: h = bf16(x + residual) (residual may be null; then h = x and
 * residual_out is unused), y = bf16(bf16(h * rsqrt(mean(h^2) + variance_epsilon))
 * * weight).  H a multiple of 128, at most 16384; rows 16-byte aligned. */
typedef struct bfp8_rmsnorm_quant_problem {
  const void* x;
  int64_t ldx;
  const void* residual;
  int64_t ldr;
  void* residual_out;
  int64_t ldro;
  const void* weight;
  void* y;
  int64_t ldy;
  void* q;
  int64_t ldq;
  float* s;
  int64_t s_m, s_k;
  int M, H;
  float variance_epsilon, eps;
} bfp8_rmsnorm_quant_problem;
int bfp8_launch_rmsnorm_quant(const bfp8_rmsnorm_quant_problem* p, void* stream);

/* SiLU-and-mul: x [M, 2I] (gate then up), y = bf16(bf16(silu(gate)) * up) of
 * shape [M, I].  I a multiple of 128; rows 16-byte aligned. */
typedef struct bfp8_silu_mul_quant_problem {
  const void* x;
  int64_t ldx;
  void* y;
  int64_t ldy;
  void* q;
  int64_t ldq;
  float* s;
  int64_t s_m, s_k;
  int M, I;
  float eps;
} bfp8_silu_mul_quant_problem;
int bfp8_launch_silu_mul_quant(const bfp8_silu_mul_quant_problem* p, void* stream);

/* The message of the last failed call on this host thread ("" if none).
 * No reference counterpart (the reference throws std::runtime_error). */
const char* bfp8_last_error(void);

/* Watchdog status of the current device: 0, or the code that the first
 * kernel whose bounded wait on a barrier gave up wrote (the kernel then
 * returned early instead of hanging).  Synchronises the device.  With
 * reset != 0 the word is cleared.  No reference counterpart. */
int64_t bfp8_device_status(int reset);

/* ABI version of this header (1). */
int bfp8_abi_version(void);

/* Roofline probes.  No counterpart in the reference.  Measure, on the current
 * device, the dense e4m3 tensor-core rate (back-to-back 128 x n x 32
 * tcgen05 MMAs from shared memory on every SM, n = 128 or 256; TFLOP/s and
 * multiply-adds per clock per SM) and the HBM read rate over a caller
 * buffer of `bytes` (16-byte aligned, larger than L2), in GB/s.  They run
 * synchronously and allocate a little scratch; not for the hot path. */
int bfp8_probe_mma(int n, int iters, double* tflops, double* macs_per_clock);
int bfp8_probe_hbm_read(const void* buf, int64_t bytes, int reps, double* gbs);
/* One K block's raw partial sums as the GEMM's tensor cores form them:
 * a [128 x 128] and b [32 x 128] e4m3 row-major device arrays (16-byte
 * aligned) -> d [128 x 32] fp32 = four K = 32 tcgen05 MMAs, unscaled, before
 * any rounding of the GEMM's own.  For measuring the MMA's accumulation. */
int bfp8_probe_block(const void* a, const void* b, float* d, void* stream);
/* Exhaustive check of the activation quantizer's arithmetic: the fast path
 * the kernels use (reciprocal times x with one correction step) against the
 * reference's sequence (one IEEE division per value), on every pair of a
 * group amax (eps or any finite bf16 magnitude) and a bf16 value up to it.
 * *mismatches = codes that differ; *first = (amax bits << 32) | (x bits + 1)
 * of the first one, 0 if none.  Synchronous; allocates a few bytes. */
int bfp8_probe_quantizer(float eps, unsigned long long* mismatches, unsigned long long* first);
/* Exhaustive check of the quantizer's scale: amax / 448 as the kernels form
 * it (a product with RN(1/448) and one correction step) against the IEEE
 * division, on every finite non-negative float amax.  *mismatches = scales
 * that differ; *first = bits + 1 of the first one, 0 if none.  Synchronous;
 * allocates a few bytes. */
int bfp8_probe_scale(unsigned long long* mismatches, unsigned long long* first);

#ifdef __cplusplus
}
#endif

#endif /* BLOCKFP8_B200_H */
