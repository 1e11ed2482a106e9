"""Autotune the B200 plan tables: time every configuration x split count on
the Qwen3-8B linear shapes and write the winners to csrc/plan_table.inc;
then, for the decode sizes, time the fused path (bf16 in) both ways --
quantization kernel + the tabulated GEMM plan, and every plan that
quantizes inside the GEMM -- and write the winners to
csrc/fused_plan_table.inc.

    python -m blockfp8_b200.autotune [--out results.json] [--write-table] [--fused-only]
    python -m blockfp8_b200.autotune --gemm-only --tp 2,4,8 --write-table   # tensor-parallel shards

Counterpart of the reference's bench/autotune.py (sweep :66-82, table
:169-177), re-done for B200: each candidate GEMM is timed by
timing.rotating_graph_us -- one CUDA graph of back-to-back launches over
weight copies that together exceed L2 -- so plans are ranked by device time
with cold weights, not by launch overhead or timer resolution.
Rebuild (python -m blockfp8_b200.build) after writing the table.
"""

import argparse
import ctypes
import json
import os

import torch

from . import _native, capi, timing

HERE = os.path.dirname(os.path.abspath(__file__))
TABLE = os.path.join(HERE, "csrc", "plan_table.inc")
FUSED_TABLE = os.path.join(HERE, "csrc", "fused_plan_table.inc")
FUSED_M = [1, 2, 4, 8, 16, 32, 64]
QUANT_KERNEL, IN_GEMM = 1, 2
LAYERS = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (24576, 4096), "down": (4096, 12288)}


def tp_layers(degrees) -> dict:
    """The same layers as one GPU of a tensor-parallel group sees them:
    qkv and gate_up split along N (column-parallel), o and down along K
    (row-parallel)."""
    out = {}
    for tp in degrees:
        for name, (n, k) in LAYERS.items():
            out[f"{name}/tp{tp}"] = (n // tp, k) if name in ("qkv", "gate_up") else (n, k // tp)
    return out
TUNE_M = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192]
SPLITS = [1, 2, 3, 4, 6, 8, 12, 16]  # and stream-K (negative) where the tiles fill waves unevenly


def candidates(m, n, k, num_configs, names, num_sms=148):
    kt = -(-k // 128)
    for config in range(num_configs):
        swap = names[config].startswith("w")
        if swap and m > 64:
            continue
        bm = int(names[config][1:].split("t" if swap else "n")[0])
        bn = int(names[config].split("t" if swap else "n")[1].split("s")[0])
        tiles = (-(-(n if swap else m) // bm)) * (-(-(m if swap else n) // bn))
        slots = num_sms // (bm // 128)  # a 256-row tile takes a CTA pair
        for splits in SPLITS:
            if splits > kt or (splits > 1 and tiles >= 2 * slots):
                continue
            per = -(-kt // splits)
            if -(-kt // per) != splits:
                continue
            yield config, splits
        if bm == 128 and tiles < 4 * num_sms and tiles % num_sms and tiles * kt >= 2 * num_sms:
            yield config, -num_sms  # stream-K: every SM the same number of K blocks


def sweep(calls=64, layers=None, ms=None, shapes=None):
    dev = torch.device("cuda", 0)
    lib = _native.capi()
    nconf = lib.bfp8_num_configs()
    names = [lib.bfp8_config_name(i).decode() for i in range(nconf)]
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    results = []
    for name, (n, k) in (shapes or LAYERS).items():
        if layers and name not in layers:
            continue
        g = torch.Generator(device=dev).manual_seed(0)
        copies = timing.copies_for(n * k)
        bs = [(torch.randn(n, k, generator=g, device=dev) * 8).clamp(-448, 448).to(torch.float8_e4m3fn)
              for _ in range(copies)]
        sbs = [torch.rand(-(-n // 128), -(-k // 128), generator=g, device=dev) * 1e-3
               for _ in range(copies)]
        for m in ms or TUNE_M:
            a = (torch.randn(m, k, generator=g, device=dev) * 8).clamp(-448, 448).to(torch.float8_e4m3fn)
            sa = torch.rand(-(-k // 128), m, generator=g, device=dev).t() * 1e-2
            c = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
            ps = [capi.problem(a, sa, bs[i], sbs[i], c) for i in range(copies)]
            n_calls = calls if m <= 512 else max(copies, calls // 8)
            timings = []
            for config, splits in candidates(m, n, k, nconf, names, sms):
                plan = _native.Plan(config, splits, 0)
                ws, cnt = capi.scratch(ps[0], plan, dev)
                us = timing.rotating_graph_us(lambda i: capi.launch_gemm(ps[i], plan, ws, cnt),
                                              copies, n_calls)
                timings.append({"config": config, "name": names[config], "splits": splits, "us": us})
            best = min(timings, key=lambda t: t["us"])
            results.append({"layer": name, "n": n, "k": k, "m": m, "best": best, "all": timings})
            print(f"{name:8s} M={m:5d}: {best['name']} x{best['splits']} {best['us']:.2f} us", flush=True)
    assert _native.device_status(reset=True) == 0
    return results, names


def sweep_fused(calls=64, layers=None, ms=None):
    """Per decode shape, the fastest fused plan: (config, splits, mode)."""
    dev = torch.device("cuda", 0)
    lib = _native.capi()
    nconf = lib.bfp8_num_configs()
    names = [lib.bfp8_config_name(i).decode() for i in range(nconf)]
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    results = []
    for name, (n, k) in LAYERS.items():
        if layers and name not in layers:
            continue
        g = torch.Generator(device=dev).manual_seed(0)
        copies = timing.copies_for(n * k)
        bs = [(torch.randn(n, k, generator=g, device=dev) * 8).clamp(-448, 448).to(torch.float8_e4m3fn)
              for _ in range(copies)]
        sbs = [torch.rand(-(-n // 128), -(-k // 128), generator=g, device=dev) * 1e-3
               for _ in range(copies)]
        for m in ms or FUSED_M:
            x = torch.randn(m, k, generator=g, device=dev).to(torch.bfloat16)
            c = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
            ps = [capi.problem(x, None, bs[i], sbs[i], c) for i in range(copies)]
            base = lib.bfp8_choose_plan(m, n, k, sms)
            plans = [(base.config, base.splits, QUANT_KERNEL)]
            for config, splits in candidates(m, n, k, nconf, names, sms):
                if not names[config].startswith("w"):
                    continue
                # in-GEMM quantization applies when the plan needs no
                # quantized-activation front in its workspace
                p_in, p_plain = _native.Plan(config, splits, IN_GEMM), _native.Plan(config, splits, 0)
                if (lib.bfp8_workspace_bytes(ctypes.byref(ps[0]), p_in)
                        == lib.bfp8_workspace_bytes(ctypes.byref(ps[0]), p_plain)):
                    plans.append((config, splits, IN_GEMM))
            timings = []
            for config, splits, mode in plans:
                plan = _native.Plan(config, splits, mode)
                ws, cnt = capi.scratch(ps[0], plan, dev)
                us = timing.rotating_graph_us(lambda i: capi.launch_gemm(ps[i], plan, ws, cnt), copies, calls)
                timings.append({"config": config, "name": names[config], "splits": splits, "mode": mode,
                                "us": us})
            best = min(timings, key=lambda t: t["us"])
            results.append({"layer": name, "n": n, "k": k, "m": m, "best": best, "all": timings})
            qk = timings[0]["us"]
            print(f"{name:8s} M={m:5d}: {best['name']} x{best['splits']} mode {best['mode']} "
                  f"{best['us']:.2f} us (quant kernel + GEMM {qk:.2f} us)", flush=True)
    assert _native.device_status(reset=True) == 0
    return results, names


def write_fused_table(results, names) -> None:
    lines = ["// Generated by blockfp8_b200/autotune.py on a B200; do not edit.",
             "// Configurations: " + ", ".join(names),
             f"// {{N, K, M, config, splits, mode}}; mode {QUANT_KERNEL} = quantization kernel + GEMM, "
             f"{IN_GEMM} = in the GEMM"]
    for r in results:
        b = r["best"]
        lines.append(f"{{{r['n']}, {r['k']}, {r['m']}, {b['config']}, {b['splits']}, {b['mode']}}},")
    with open(FUSED_TABLE, "w") as f:
        f.write("\n".join(lines) + "\n")


def read_table(path=None) -> dict:
    """{(n, k, m): (config, splits)} of a generated plan_table.inc (TABLE by default)."""
    rows = {}
    for line in open(path or TABLE):
        line = line.strip()
        if line.startswith("{") and line.endswith("},"):
            n, k, m, config, splits = (int(v) for v in line[1:-2].split(","))
            rows[(n, k, m)] = (config, splits)
    return rows


def write_table(results, names, merge=True) -> None:
    """Write the winners; with merge, rows of shapes not in `results` stay."""
    rows = read_table(TABLE) if merge and os.path.exists(TABLE) else {}
    for r in results:
        rows[(r["n"], r["k"], r["m"])] = (r["best"]["config"], r["best"]["splits"])
    order = {shape: i for i, shape in enumerate(list(LAYERS.values()) + list(tp_layers((2, 4, 8)).values()))}
    lines = ["// Generated by blockfp8_b200/autotune.py on a B200; do not edit.",
             "// Configurations: " + ", ".join(names),
             "// {N, K, M, config, splits}; splits < 0: stream-K over -splits CTAs"]
    for (n, k, m), (config, splits) in sorted(rows.items(), key=lambda t: (order.get(t[0][:2], 99), t[0])):
        lines.append(f"{{{n}, {k}, {m}, {config}, {splits}}},")
    with open(TABLE, "w") as f:
        f.write("\n".join(lines) + "\n")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    ap.add_argument("--calls", type=int, default=64)
    ap.add_argument("--write-table", action="store_true")
    ap.add_argument("--fused-only", action="store_true", help="keep plan_table.inc; tune the fused table")
    ap.add_argument("--gemm-only", action="store_true", help="tune plan_table.inc only")
    ap.add_argument("--ms", type=str, default=None, help="comma-separated M values of the GEMM sweep")
    ap.add_argument("--tp", type=str, default=None,
                    help="comma-separated tensor-parallel degrees: sweep their shard shapes instead")
    args = ap.parse_args()
    out = {}
    if not args.fused_only:
        ms = [int(v) for v in args.ms.split(",")] if args.ms else None
        shapes = tp_layers([int(v) for v in args.tp.split(",")]) if args.tp else None
        results, names = sweep(args.calls, ms=ms, shapes=shapes)
        out.update(configs=names, results=results)
        if args.write_table:
            write_table(results, names)
    if not args.gemm_only:  # after a GEMM sweep, rebuild first: mode 1 uses the compiled table
        fused, names = sweep_fused(args.calls)
        out.update(configs=names, fused=fused)
        if args.write_table:
            write_fused_table(fused, names)
    if args.out:
        with open(args.out, "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
