"""End-to-end vLLM on B200: stock vLLM against vLLM with the blockfp8 plugin.

The model is a random-init decoder with the Qwen3-8B architecture: 36
layers, hidden 4096, 32 query / 8 key-value heads of 128, SwiGLU 12288,
vocab 151936. Every linear layer holds e4m3 weights with one fp32 scale
per 128x128 block, drawn as N(0, 0.02) and then quantized. The model
directory holds only a config.json with those numbers and a 128x128
block-FP8 quantization_config; there is no tokenizer (token-id prompts)
and no checkpoint (load_format "dummy"). Workload (the reference's
bench/e2e_vllm.py:132-211 on a random model):

  prefill   16 prompts of 1024 uniform-random token ids, max_tokens=1,
            prefix caching off; prompt tokens / wall time.
  decode    batch B in {1, 16} of 1024-token prompts, generated with
            ignore_eos to 1 and to 129 tokens; TPOT = difference / 128
            (the prefill cancels).
  outputs   greedy continuations of 4 fixed prompts with their logprobs.
            Every later configuration also scores the first one's
            continuation (prompt_logprobs), so all score the same tokens.

Configurations (--impls, in the order given; the first is the output
anchor):

  triton    vLLM's Triton block-FP8 kernel (linear_backend="triton"):
            fp32 scales, the reference's numerics.
  stock     vLLM's own choice on sm_100: its vendored DeepGEMM, which
            rounds weight and activation scales up to powers of two (UE8M0).
  cutlass   vLLM's CUTLASS block-FP8 kernel (linear_backend="cutlass"),
            fp32 scales.
  plugin    the blockfp8 plugin (BlockFp8LinearKernel).

Each figure is the median of --reps repetitions after one warm-up. Each
configuration runs in its own process (a fresh engine, nothing shared).
vLLM finds plugins through the "vllm.general_plugins" entry points of
installed distributions. Nothing is installed: each run puts a throwaway
.dist-info directory on PYTHONPATH that declares two of them:

  blockfp8              blockfp8_vllm:register (the plugin; plugin run only)
  blockfp8_e2e_weights  blockfp8_vllm.e2e:install_weight_init (every run)

    python -m blockfp8_vllm.e2e --tp 1 --out results.json
"""

from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# Qwen3-8B architecture (the model numbers the benchmark configuration names)
QWEN3_8B = {
    "architectures": ["Qwen3ForCausalLM"],
    "model_type": "qwen3",
    "hidden_size": 4096,
    "intermediate_size": 12288,
    "num_hidden_layers": 36,
    "num_attention_heads": 32,
    "num_key_value_heads": 8,
    "head_dim": 128,
    "vocab_size": 151936,
    "max_position_embeddings": 40960,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "hidden_act": "silu",
    "attention_bias": False,
    "tie_word_embeddings": False,
    "torch_dtype": "bfloat16",
    "bos_token_id": 151643,
    "eos_token_id": 151645,
    "quantization_config": {
        "quant_method": "fp8",
        "activation_scheme": "dynamic",
        "fmt": "e4m3",
        "weight_block_size": [128, 128],
    },
}

PREFILL_PROMPTS, PREFILL_LEN = 16, 1024
DECODE_BATCHES = (1, 16)
DECODE_LEN = 1024
DECODE_STEPS = (1, 129)
CHECK_PROMPTS, CHECK_LEN, CHECK_TOKENS = 4, 64, 32
WEIGHT_STD = 0.02
ENGINE = dict(load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16", seed=0,
              max_model_len=4096, max_num_batched_tokens=16384, max_num_seqs=64,
              enable_prefix_caching=False, gpu_memory_utilization=0.6)
# configuration -> (extra engine arguments, the linear kernel it must select)
IMPLS = {
    "triton": ({"linear_backend": "triton"}, "TritonFp8BlockScaledMMKernel"),
    "stock": ({}, None),
    "cutlass": ({"linear_backend": "cutlass"}, "CutlassFp8BlockScaledMMKernel"),
    "plugin": ({}, "BlockFp8LinearKernel"),
}
ENTRY_POINTS = {
    "blockfp8": "blockfp8_vllm:register",
    "blockfp8_e2e_weights": "blockfp8_vllm.e2e:install_weight_init",
}


def write_model_dir(path: str) -> str:
    """config.json of the random Qwen3-8B-architecture block-FP8 model."""
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(QWEN3_8B, f, indent=1)
    return path


def write_entry_points(path: str) -> str:
    """A .dist-info under `path` that declares ENTRY_POINTS in the
    vllm.general_plugins group; importlib.metadata finds it once `path` is
    on sys.path."""
    info = os.path.join(path, "blockfp8_e2e-0.0.dist-info")
    os.makedirs(info, exist_ok=True)
    with open(os.path.join(info, "METADATA"), "w") as f:
        f.write("Metadata-Version: 2.1\nName: blockfp8-e2e\nVersion: 0.0\n")
    with open(os.path.join(info, "entry_points.txt"), "w") as f:
        f.write("[vllm.general_plugins]\n")
        for name, target in ENTRY_POINTS.items():
            f.write(f"{name} = {target}\n")
    return path


# ---- weights: runs inside every vLLM process -----------------------------------------

_seed = [0]


def init_module_weights(module) -> int:
    """Random init of one module's own parameters, the usual decoder
    initialization: block-FP8 linear weights N(0, WEIGHT_STD) quantized to e4m3
    with 128x128 block scales; other 2-D floating weights (embedding, LM head)
    N(0, WEIGHT_STD); 1-D weights (RMSNorm) one. Returns the number of
    tensors set."""
    import torch

    from blockfp8_b200 import FP8_DTYPE, quantize_weights

    params = dict(module.named_parameters(recurse=False))
    done = 0
    w = params.get("weight")
    if w is None:
        return 0
    _seed[0] += 1
    gen = torch.Generator(device=w.device).manual_seed(_seed[0])
    with torch.no_grad():
        scale = params.get("weight_scale_inv")
        if w.dtype == FP8_DTYPE and scale is not None and w.dim() == 2:
            wq, ws = quantize_weights(torch.randn(w.shape, generator=gen, device=w.device) * WEIGHT_STD)
            if tuple(ws.shape) != tuple(scale.shape):
                raise RuntimeError(f"block scales {tuple(scale.shape)} for weight {tuple(w.shape)}")
            w.copy_(wq)
            scale.copy_(ws)
            done = 2
        elif w.is_floating_point() and w.dim() == 2:
            w.copy_(torch.randn(w.shape, generator=gen, device=w.device) * WEIGHT_STD)
            done = 1
        elif w.is_floating_point() and w.dim() == 1:
            w.fill_(1.0)
            done = 1
    return done


def install_weight_init() -> None:
    """Entry point: after vLLM's dummy loader fills a module with its uniform
    +-1e-3 values, give the module's own weights init_module_weights'. The
    loader visits parents before children, so every module's own call is
    the last to touch its parameters."""
    from vllm.model_executor.model_loader import dummy_loader

    original = dummy_loader.initialize_dummy_weights
    if getattr(original, "blockfp8_e2e", False):
        return

    def initialize(model, *args, **kwargs):
        original(model, *args, **kwargs)
        init_module_weights(model)

    initialize.blockfp8_e2e = True
    dummy_loader.initialize_dummy_weights = initialize


def linear_kernels(worker) -> list[str]:
    """Names of the block-FP8 linear kernels vLLM selected (collective_rpc)."""
    model = worker.model_runner.get_model()
    names = set()
    for m in model.modules():
        kernel = getattr(getattr(m, "quant_method", None), "fp8_linear", None)
        if kernel is not None:
            names.add(type(kernel).__name__)
    return sorted(names)


# ---- one configuration (a subprocess) --------------------------------------------------

def _prompts(n: int, length: int, seed: int):
    from vllm.inputs import TokensPrompt

    rng = random.Random(seed)
    return [TokensPrompt(prompt_token_ids=[rng.randrange(1000, 150000) for _ in range(length)])
            for _ in range(n)]


def _median_s(fn, reps: int) -> tuple[float, list[float]]:
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), times


def run_config(impl: str, tp: int, reps: int, reference: dict | None) -> dict:
    import torch
    import vllm
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    model_dir = write_model_dir(tempfile.mkdtemp(prefix="qwen3-8b-arch-"))
    t0 = time.perf_counter()
    engine = {**ENGINE, **IMPLS[impl][0]}
    llm = LLM(model=model_dir, tensor_parallel_size=tp, **engine)
    out = {"impl": impl, "tp": tp, "vllm": vllm.__version__, "torch": torch.__version__,
           "device": torch.cuda.get_device_name(0), "engine": engine, "reps": reps,
           "load_s": time.perf_counter() - t0,
           "linear_kernels": sorted(set(sum(llm.collective_rpc(linear_kernels), [])))}

    prompts = _prompts(PREFILL_PROMPTS, PREFILL_LEN, seed=1)
    one = SamplingParams(max_tokens=1, temperature=0.0, ignore_eos=True, detokenize=False)
    llm.generate(prompts, one, use_tqdm=False)
    s, reps_s = _median_s(lambda: llm.generate(prompts, one, use_tqdm=False), reps)
    tokens = PREFILL_PROMPTS * PREFILL_LEN
    out["prefill"] = {"prompts": PREFILL_PROMPTS, "prompt_len": PREFILL_LEN, "tokens": tokens,
                      "s": s, "s_reps": reps_s, "tokens_per_s": tokens / s}
    print(f"[{impl} tp{tp}] prefill {PREFILL_PROMPTS}x{PREFILL_LEN}: {tokens / s:.0f} tok/s", flush=True)

    out["decode"] = []
    for batch in DECODE_BATCHES:
        prompts = _prompts(batch, DECODE_LEN, seed=100 + batch)
        short, long_ = (SamplingParams(max_tokens=n, temperature=0.0, ignore_eos=True, detokenize=False)
                        for n in DECODE_STEPS)
        llm.generate(prompts, long_, use_tqdm=False)
        t_short, r_short = _median_s(lambda: llm.generate(prompts, short, use_tqdm=False), reps)
        t_long, r_long = _median_s(lambda: llm.generate(prompts, long_, use_tqdm=False), reps)
        tpot = (t_long - t_short) / (DECODE_STEPS[1] - DECODE_STEPS[0])
        out["decode"].append({"batch": batch, "prompt_len": DECODE_LEN, "max_tokens": DECODE_STEPS,
                              "s_short": t_short, "s_long": t_long, "s_short_reps": r_short,
                              "s_long_reps": r_long, "tpot_ms": tpot * 1e3})
        print(f"[{impl} tp{tp}] decode B={batch}: TPOT {tpot * 1e3:.3f} ms", flush=True)

    check = _prompts(CHECK_PROMPTS, CHECK_LEN, seed=7)
    greedy = llm.generate(check, SamplingParams(max_tokens=CHECK_TOKENS, temperature=0.0, ignore_eos=True,
                                                logprobs=0, detokenize=False), use_tqdm=False)
    out["greedy"] = [{"tokens": list(o.outputs[0].token_ids),
                      "logprobs": [lp[t].logprob for t, lp in zip(o.outputs[0].token_ids, o.outputs[0].logprobs)]}
                     for o in greedy]
    if reference is not None:
        forced_in = [TokensPrompt(prompt_token_ids=list(p["prompt_token_ids"]) + r["tokens"])
                     for p, r in zip(check, reference["greedy"])]
        forced = llm.generate(forced_in, SamplingParams(max_tokens=1, temperature=0.0, prompt_logprobs=0,
                                                        detokenize=False), use_tqdm=False)
        out["teacher_forced"] = [[lp[t].logprob for t, lp in zip(r["tokens"], o.prompt_logprobs[CHECK_LEN:])]
                                 for r, o in zip(reference["greedy"], forced)]
    llm.llm_engine.engine_core.shutdown()
    return out


def compare(anchor: dict, other: dict) -> dict:
    """Agreement of one configuration's outputs with the anchor run's: how
    many greedy tokens agree before the first difference, and the logprobs
    `other` gives the anchor's tokens against the anchor's own."""
    first_diff = []
    for s, p in zip(anchor["greedy"], other["greedy"]):
        same = [a == b for a, b in zip(s["tokens"], p["tokens"])]
        first_diff.append(same.index(False) if False in same else len(same))
    deltas = [abs(a - b) for s, t in zip(anchor["greedy"], other.get("teacher_forced", []))
              for a, b in zip(s["logprobs"], t)]
    return {"greedy_tokens_agreeing": first_diff,
            "teacher_forced_logprob_abs_diff_max": max(deltas) if deltas else None,
            "teacher_forced_logprob_abs_diff_mean": statistics.fmean(deltas) if deltas else None}


# ---- driver --------------------------------------------------------------------------

def _spawn(impl: str, args, reference_path: str | None, out_path: str, plugins_dir: str) -> dict:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([ROOT, plugins_dir] + ([env["PYTHONPATH"]] if env.get("PYTHONPATH") else []))
    env["VLLM_PLUGINS"] = "blockfp8,blockfp8_e2e_weights" if impl == "plugin" else "blockfp8_e2e_weights"
    env["VLLM_LOGGING_LEVEL"] = env.get("VLLM_LOGGING_LEVEL", "INFO")
    env["VLLM_ALLOW_INSECURE_SERIALIZATION"] = "1"  # collective_rpc(linear_kernels)
    env.setdefault("NCCL_NVLS_ENABLE", "0")
    cmd = [sys.executable, "-m", "blockfp8_vllm.e2e", "--worker", impl, "--tp", str(args.tp),
           "--reps", str(args.reps), "--result", out_path]
    if reference_path:
        cmd += ["--reference", reference_path]
    subprocess.run(cmd, env=env, check=True, timeout=args.timeout)
    with open(out_path) as f:
        return json.load(f)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--impls", default="triton,stock,cutlass,plugin",
                    help="comma-separated configurations from " + ", ".join(IMPLS) + "; the first anchors the outputs")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--timeout", type=int, default=1500, help="seconds per configuration")
    ap.add_argument("--out", default=None)
    ap.add_argument("--worker", choices=tuple(IMPLS), default=None, help=argparse.SUPPRESS)
    ap.add_argument("--result", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--reference", default=None, help=argparse.SUPPRESS)
    args = ap.parse_args(argv)

    if args.worker:
        reference = None
        if args.reference:
            with open(args.reference) as f:
                reference = json.load(f)
        res = run_config(args.worker, args.tp, args.reps, reference)
        with open(args.result, "w") as f:
            json.dump(res, f)
        sys.stdout.flush()
        os._exit(0)  # vLLM's interpreter teardown can abort after the engine has stopped

    impls = args.impls.split(",")
    unknown = [i for i in impls if i not in IMPLS]
    if unknown or len(set(impls)) != len(impls):
        raise SystemExit(f"--impls: unknown or repeated configurations in {impls}")
    work = tempfile.mkdtemp(prefix="blockfp8-e2e-")
    plugins_dir = write_entry_points(os.path.join(work, "site"))
    results, anchor_path = {}, None
    for impl in impls:
        path = os.path.join(work, f"{impl}.json")
        results[impl] = _spawn(impl, args, anchor_path, path, plugins_dir)
        anchor_path = anchor_path or path
        want = IMPLS[impl][1]
        if want is not None and results[impl]["linear_kernels"] != [want]:
            raise SystemExit(f"{impl} run selected {results[impl]['linear_kernels']}, not {want}")
    agreement = {impl: compare(results[impls[0]], results[impl]) for impl in impls[1:]}
    summary = {impl: {"linear_kernels": r["linear_kernels"],
                      "prefill_tokens_per_s": round(r["prefill"]["tokens_per_s"]),
                      "tpot_ms": {str(d["batch"]): round(d["tpot_ms"], 3) for d in r["decode"]}}
               for impl, r in results.items()}
    results["agreement"] = {"anchor": impls[0], **agreement}
    summary["agreement"] = results["agreement"]
    print(json.dumps({"tp": args.tp, **summary}), flush=True)
    if args.out:
        with open(args.out, "w") as f:
            json.dump(results, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
