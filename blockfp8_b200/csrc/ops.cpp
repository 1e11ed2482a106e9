// torch.ops.blockfp8: the seven operators of the reference's extension
// (simon-jd/blockfp8 csrc/ops.cpp:213-232) -- the same schemas, defaults and
// CUDA dispatch -- implemented over the C ABI of libblockfp8_b200.so
// (include/blockfp8_b200.h).  This file is glue: tensor checks, output
// allocation, plan resolution and scratch; the kernels, planner and launch
// logic live behind the ABI.
//
// Conventions:
// - outputs are allocated on the input's device (C; q and M-major scales);
//   inputs are borrowed, never copied;
// - everything is enqueued on the current CUDA stream under a device guard
//   and nothing synchronises;
// - split-K workspace comes from the caching allocator per call (so it is
//   graph-pool memory under capture); arrival counters come from a
//   per-device pool that is zero between launches (the kernels reset what
//   they use) and is never freed, because captured graphs keep pointing at
//   it.  Two calls running at once on different streams of one device must
//   not share a pool: the ops assume one stream per device, as vLLM uses.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <deque>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "blockfp8_b200.h"

namespace {

constexpr double kDefaultEps = 1e-10;

// ---- checks ------------------------------------------------------------------
// Messages read "blockfp8[.op]: what"; callers (and the tests) match on the
// `what` part.

[[noreturn]] void reject(const char* op, const std::string& what) {
  TORCH_CHECK(false, op, ": ", what);
}

void require(bool ok, const char* op, const char* what) {
  if (!ok) reject(op, what);
}

void require_abi(int status) {
  if (status < 0) TORCH_CHECK(false, bfp8_last_error());
}

bool aligned16(const at::Tensor& t) { return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0; }

bool row_major(const at::Tensor& t, int64_t row_multiple) {
  return t.stride(1) == 1 && t.stride(0) % row_multiple == 0;
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Weights and their 128x128 block scales, for a reduction length K.
void check_weights(const at::Tensor& b, const at::Tensor& b_scales, int64_t K) {
  const char* op = "blockfp8";
  require(b.is_cuda() && b_scales.is_cuda(), op, "all operands must be CUDA tensors");
  require(b.scalar_type() == at::kFloat8_e4m3fn, op, "b must be float8_e4m3fn");
  require(b_scales.scalar_type() == at::kFloat, op, "scales must be float32");
  require(b.dim() == 2 && b.size(1) == K, op, "bad shapes");
  require(K > 0 && K % 16 == 0, op, "K must be a positive multiple of 16");
  require(b.size(0) > 0 && b.size(0) % 8 == 0, op, "N must be a positive multiple of 8");
  require(row_major(b, 16), op, "b must be row-major with 16-element aligned rows");
  require(aligned16(b), op, "b must be 16-byte aligned");
  require(b_scales.dim() == 2 && b_scales.size(0) == cdiv(b.size(0), 128) && b_scales.size(1) == cdiv(K, 128), op,
          "b_scales must be [ceil(N/128), ceil(K/128)]");
  require(b.device() == b_scales.device(), op, "all operands must be on one device");
  require(b.size(0) <= INT32_MAX && K <= INT32_MAX, op, "too large");
}

// bf16 activations of linear / quantize.
void check_activations(const at::Tensor& x, const char* op) {
  require(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2, op,
          "x must be a 2-D bfloat16 CUDA tensor");
  require(row_major(x, 8) && aligned16(x), op, "x must be row-major with 16-byte aligned rows");
  require(x.size(1) > 0 && x.size(1) % 16 == 0, op, "K must be a positive multiple of 16");
  require(x.size(0) <= INT32_MAX && x.size(1) <= INT32_MAX, op, "too large");
}

// ---- split-K arrival counters --------------------------------------------------

class CounterPool {
 public:
  // At least `needed` zeroed ints on `device`.
  int* get(const at::Device& device, int needed) {
    std::lock_guard<std::mutex> lock(mu_);
    at::Tensor& live = live_[device.index()];
    if (!live.defined() || live.numel() < needed) {
      if (live.defined()) kept_.push_back(live);  // a captured graph may still use it
      int64_t size = int64_t(1) << 16;
      while (size < needed) size *= 2;
      live = at::zeros({size}, at::TensorOptions().dtype(at::kInt).device(device));
    }
    return live.data_ptr<int>();
  }

 private:
  std::mutex mu_;
  std::map<int, at::Tensor> live_;
  std::deque<at::Tensor> kept_;
};

CounterPool& counter_pool() {
  static CounterPool pool;
  return pool;
}

// ---- plans and launches ----------------------------------------------------------

int sm_count() { return at::cuda::getCurrentDeviceProperties()->multiProcessorCount; }

// The plan a call runs: the library's choice, unless the caller names a
// configuration (then split_k defaults to one split) and/or a split count
// (> 0: K splits; < 0: stream-K over -split_k CTAs).
bfp8_plan resolve(bfp8_plan chosen, int64_t config, int64_t split_k, int num_configs) {
  if (config >= 0) {
    TORCH_CHECK(config < num_configs, "blockfp8: config out of range");
    chosen.config = int(config);
    if (split_k == 0) split_k = 1;
  }
  if (split_k != 0) chosen.splits = int(split_k);
  return chosen;
}

// Scratch for one launch (workspace from the caching allocator, counters
// from the pool), then the launch on the current stream.
void launch(const bfp8_gemm_problem& p, const bfp8_plan& plan, const at::Tensor& like) {
  const int64_t ws_bytes = bfp8_workspace_bytes(&p, plan);
  require_abi(int(std::min<int64_t>(ws_bytes, 0)));
  const int n_counters = bfp8_counters_needed(&p, plan);
  require_abi(std::min(n_counters, 0));
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({cdiv(ws_bytes, 4)}, like.options().dtype(at::kFloat));
  int* counters = n_counters > 0 ? counter_pool().get(like.device(), n_counters) : nullptr;
  require_abi(bfp8_launch_gemm(&p, plan, ws.defined() ? ws.data_ptr<float>() : nullptr, counters,
                               at::cuda::getCurrentCUDAStream().stream()));
}

// The weight side and output of a problem; the caller fills in A.
bfp8_gemm_problem weight_problem(const at::Tensor& b, const at::Tensor& b_scales, const at::Tensor& c) {
  bfp8_gemm_problem p{};
  p.b = b.data_ptr();
  p.ldb = b.stride(0);
  p.sb = b_scales.data_ptr<float>();
  p.sb_n = b_scales.stride(0);
  p.sb_k = b_scales.stride(1);
  p.c = c.data_ptr();
  p.ldc = c.stride(0);
  p.M = int(c.size(0));
  p.N = int(b.size(0));
  p.K = int(b.size(1));
  p.eps = float(kDefaultEps);
  return p;
}

// ---- the operators -------------------------------------------------------------

// C = (a, a_scales) x (b, b_scales)^T: e4m3 activations with per-row 1x128
// scales (any strides) against 128x128-block-scaled e4m3 weights, bf16 out.
at::Tensor gemm(const at::Tensor& a, const at::Tensor& a_scales, const at::Tensor& b, const at::Tensor& b_scales,
                int64_t config, int64_t split_k) {
  const char* op = "blockfp8.gemm";
  require(a.is_cuda() && a_scales.is_cuda(), op, "all operands must be CUDA tensors");
  require(a.scalar_type() == at::kFloat8_e4m3fn, op, "a must be float8_e4m3fn");
  require(a_scales.scalar_type() == at::kFloat, op, "scales must be float32");
  require(a.dim() == 2, op, "bad shapes");
  check_weights(b, b_scales, a.size(1));
  require(row_major(a, 16), op, "a must be row-major with 16-element aligned rows");
  require(aligned16(a), op, "a must be 16-byte aligned");
  require(a_scales.dim() == 2 && a_scales.size(0) == a.size(0) && a_scales.size(1) == cdiv(a.size(1), 128), op,
          "a_scales must be [M, ceil(K/128)]");
  require(a.device() == b.device() && a.device() == a_scales.device(), op, "all operands must be on one device");
  require(a.size(0) <= INT32_MAX, op, "too large");

  const at::cuda::CUDAGuard guard(a.device());
  at::Tensor c = at::empty({a.size(0), b.size(0)}, a.options().dtype(at::kBFloat16));
  if (c.size(0) == 0) return c;
  bfp8_gemm_problem p = weight_problem(b, b_scales, c);
  p.a = a.data_ptr();
  p.lda = a.stride(0);
  p.sa = a_scales.data_ptr<float>();
  p.sa_m = a_scales.stride(0);
  p.sa_k = a_scales.stride(1);
  launch(p, resolve(bfp8_choose_plan(p.M, p.N, p.K, sm_count()), config, split_k, bfp8_num_configs()), a);
  return c;
}

// The same product from bf16 activations, quantized as part of the call
// (bitwise gemm(quantize(x))).
at::Tensor gemm_bf16(const at::Tensor& x, const at::Tensor& b, const at::Tensor& b_scales, int64_t config,
                     int64_t split_k, double eps) {
  const char* op = "blockfp8.gemm_bf16";
  require(x.is_cuda(), op, "all operands must be CUDA tensors");
  require(x.scalar_type() == at::kBFloat16, op, "x must be bfloat16");
  require(x.dim() == 2, op, "bad shapes");
  check_weights(b, b_scales, x.size(1));
  require(row_major(x, 8), op, "x must be row-major with 8-element aligned rows");
  require(aligned16(x), op, "x must be 16-byte aligned");
  require(x.device() == b.device(), op, "all operands must be on one device");
  require(x.size(0) <= INT32_MAX, op, "too large");
  require(eps > 0, op, "eps must be positive");

  const at::cuda::CUDAGuard guard(x.device());
  at::Tensor c = at::empty({x.size(0), b.size(0)}, x.options().dtype(at::kBFloat16));
  if (c.size(0) == 0) return c;
  bfp8_gemm_problem p = weight_problem(b, b_scales, c);
  p.a = x.data_ptr();
  p.lda = x.stride(0);
  p.eps = float(eps);
  launch(p, resolve(bfp8_choose_fused_plan(p.M, p.N, p.K, sm_count()), config, split_k, bfp8_num_fused_configs()),
         x);
  return c;
}

// x [M, K] bf16 -> (q [M, K] e4m3, scales [M, ceil(K/128)] float32 stored
// M-contiguous, strides (1, M)).
std::tuple<at::Tensor, at::Tensor> quantize(const at::Tensor& x, double eps) {
  const char* op = "blockfp8.quantize";
  check_activations(x, op);
  require(eps > 0, op, "eps must be positive");
  const at::cuda::CUDAGuard guard(x.device());
  const int64_t M = x.size(0), K = x.size(1);
  at::Tensor q = at::empty({M, K}, x.options().dtype(at::kFloat8_e4m3fn));
  at::Tensor s = at::empty({cdiv(K, 128), M}, x.options().dtype(at::kFloat)).t();
  const bfp8_quant_problem p{x.data_ptr(), x.stride(0), q.data_ptr(), q.stride(0), s.data_ptr<float>(),
                             s.stride(0),  s.stride(1), int(M),     int(K),      float(eps)};
  require_abi(bfp8_launch_quantize(&p, at::cuda::getCurrentCUDAStream().stream()));
  return {q, s};
}

bool prefers_fused(int64_t M, int64_t N, int64_t K) { return bfp8_prefers_fused(int(M), int(N), int(K)) != 0; }

// A linear layer on bf16 activations: the fused path where the library
// prefers it (everywhere today), else quantize() then gemm().
at::Tensor linear(const at::Tensor& x, const at::Tensor& b, const at::Tensor& b_scales) {
  check_activations(x, "blockfp8.linear");
  if (prefers_fused(x.size(0), b.size(0), x.size(1))) return gemm_bf16(x, b, b_scales, -1, 0, kDefaultEps);
  const auto qs = quantize(x, kDefaultEps);
  return gemm(std::get<0>(qs), std::get<1>(qs), b, b_scales, -1, 0);
}

// ";"-joined configuration names.
std::string joined(int count, const char* (*name_of)(int)) {
  std::string out;
  for (int i = 0; i < count; ++i) out.append(i ? ";" : "").append(name_of(i));
  return out;
}

std::string config_names() { return joined(bfp8_num_configs(), bfp8_config_name); }
std::string fused_config_names() { return joined(bfp8_num_fused_configs(), bfp8_fused_config_name); }

// ---- producers that emit the linear's operand (torch.ops.blockfp8_b200) ---------
// Not in the reference's extension: an RMSNorm and a SiLU-and-mul whose
// outputs are the e4m3 codes and M-major scales blockfp8.gemm takes, so the
// linear after them needs no quantization launch.

std::tuple<at::Tensor, at::Tensor> quant_outputs(const at::Tensor& like, int64_t M, int64_t cols) {
  at::Tensor q = at::empty({M, cols}, like.options().dtype(at::kFloat8_e4m3fn));
  at::Tensor s = at::empty({cdiv(cols, 128), M}, like.options().dtype(at::kFloat)).t();
  return {q, s};
}

// (q, scales, h): h = x + residual in bf16 when a residual is given (the
// next layer's residual), else an empty tensor.
std::tuple<at::Tensor, at::Tensor, at::Tensor> rms_norm_quant(const at::Tensor& x, const at::Tensor& weight,
                                                              double variance_epsilon,
                                                              const c10::optional<at::Tensor>& residual, double eps) {
  const char* op = "blockfp8_b200.rms_norm_quant";
  check_activations(x, op);
  const int64_t M = x.size(0), H = x.size(1);
  require(H % 128 == 0 && H <= 16384, op, "hidden size must be a multiple of 128, at most 16384");
  require(weight.is_cuda() && weight.scalar_type() == at::kBFloat16 && weight.dim() == 1 && weight.size(0) == H &&
              weight.stride(0) == 1 && aligned16(weight) && weight.device() == x.device(),
          op, "weight must be a contiguous bfloat16 [H] tensor on x's device");
  require(eps > 0 && variance_epsilon >= 0, op, "eps must be positive");
  const at::cuda::CUDAGuard guard(x.device());
  auto [q, s] = quant_outputs(x, M, H);
  at::Tensor h;
  bfp8_rmsnorm_quant_problem p{};
  p.x = x.data_ptr();
  p.ldx = x.stride(0);
  if (residual.has_value()) {
    const at::Tensor& r = *residual;
    check_activations(r, op);
    require(r.sizes() == x.sizes() && r.device() == x.device(), op, "residual must match x");
    h = at::empty({M, H}, x.options());
    p.residual = r.data_ptr();
    p.ldr = r.stride(0);
    p.residual_out = h.data_ptr();
    p.ldro = h.stride(0);
  } else {
    h = at::empty({0}, x.options());
  }
  if (M == 0) return {q, s, h};
  p.weight = weight.data_ptr();
  p.q = q.data_ptr();
  p.ldq = q.stride(0);
  p.s = s.data_ptr<float>();
  p.s_m = s.stride(0);
  p.s_k = s.stride(1);
  p.M = int(M);
  p.H = int(H);
  p.variance_epsilon = float(variance_epsilon);
  p.eps = float(eps);
  require_abi(bfp8_launch_rmsnorm_quant(&p, at::cuda::getCurrentCUDAStream().stream()));
  return {q, s, h};
}

std::tuple<at::Tensor, at::Tensor> silu_mul_quant(const at::Tensor& x, double eps) {
  const char* op = "blockfp8_b200.silu_mul_quant";
  check_activations(x, op);
  const int64_t M = x.size(0), I = x.size(1) / 2;
  require(x.size(1) % 256 == 0, op, "x must be [M, 2I] with I a multiple of 128");
  require(M <= 65535, op, "at most 65535 rows");
  require(eps > 0, op, "eps must be positive");
  const at::cuda::CUDAGuard guard(x.device());
  auto [q, s] = quant_outputs(x, M, I);
  if (M == 0) return {q, s};
  bfp8_silu_mul_quant_problem p{};
  p.x = x.data_ptr();
  p.ldx = x.stride(0);
  p.q = q.data_ptr();
  p.ldq = q.stride(0);
  p.s = s.data_ptr<float>();
  p.s_m = s.stride(0);
  p.s_k = s.stride(1);
  p.M = int(M);
  p.I = int(I);
  p.eps = float(eps);
  require_abi(bfp8_launch_silu_mul_quant(&p, at::cuda::getCurrentCUDAStream().stream()));
  return {q, s};
}

}  // namespace

TORCH_LIBRARY(blockfp8_b200, m) {
  m.def("rms_norm_quant(Tensor x, Tensor weight, float variance_epsilon, Tensor? residual=None, "
        "float eps=1e-10) -> (Tensor, Tensor, Tensor)");
  m.def("silu_mul_quant(Tensor x, float eps=1e-10) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(blockfp8_b200, CUDA, m) {
  m.impl("rms_norm_quant", &rms_norm_quant);
  m.impl("silu_mul_quant", &silu_mul_quant);
}

TORCH_LIBRARY(blockfp8, m) {
  m.def("gemm(Tensor a, Tensor a_scales, Tensor b, Tensor b_scales, int config=-1, int split_k=0) -> Tensor");
  m.def(
      "gemm_bf16(Tensor x, Tensor b, Tensor b_scales, int config=-1, int split_k=0, float eps=1e-10) -> Tensor");
  m.def("quantize(Tensor x, float eps=1e-10) -> (Tensor, Tensor)");
  m.def("linear(Tensor x, Tensor b, Tensor b_scales) -> Tensor");
  m.def("prefers_fused(int m, int n, int k) -> bool", &prefers_fused);
  m.def("config_names() -> str", &config_names);
  m.def("fused_config_names() -> str", &fused_config_names);
}

TORCH_LIBRARY_IMPL(blockfp8, CUDA, m) {
  m.impl("gemm", &gemm);
  m.impl("gemm_bf16", &gemm_bf16);
  m.impl("quantize", &quantize);
  m.impl("linear", &linear);
}
