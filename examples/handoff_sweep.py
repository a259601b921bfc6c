#!/usr/bin/env python
"""KV-handoff microbenchmark over request sizes and compression modes.

Reproduces the sweep of the reference's handoff microbenchmark: synthetic
bf16 KV per request from about 1 MB to 4 GB raw (Qwen2.5-7B KV shapes: 28
layers, 4 KV heads, head_dim 128, so a request of T tokens holds T x 57,344
bytes), N(0,1) with 3% outlier key channels x12, paged in 16-token blocks at
shuffled block ids, for compression off and hybrid_ratio 0 / 0.3 / 1.0 of
the default mode.  Every point is one request per step, device-timed with
CUDA events between barriers, the maximum over ranks.

* 1 GPU: compress -> decompress round trip (or raw gather -> scatter);
* N >= 2 GPUs (torchrun, one rank per GPU): pairs r <-> r + N/2, the
  producer's kernels store into the consumer's receive ring over NVLink
  (times are per pair).

``--impl reference`` (or ``both``) also runs the unmodified reference from
``baseline/_ref`` through its public adapter and NCCL transport on the same
workload; its pipeline is slow on the largest requests, so
``--max-reference-tokens`` bounds its sizes.

Usage::

    python examples/handoff_sweep.py --impl both --out sweep_1gpu.md
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/handoff_sweep.py \\
        --gpus 2 --impl both --out sweep_2gpu.md
"""

from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

BYTES_PER_TOKEN = 28 * 2 * 4 * 128 * 2  # Qwen2.5-7B KV, bf16
DEFAULT_TOKENS = [16, 256, 4096, 16384, 74912]  # 0.9 MB ... 4.0 GiB per request
MODES = {"off": ("off", None), "h0": ("default", 0.0), "h0.3": ("default", 0.3),
         "h1": ("default", 1.0)}


def steps_for(tokens: int, budget_bytes: float = 2e9, lo: int = 3, hi: int = 40) -> int:
    """Timed steps for a request size: about ``budget_bytes`` of raw KV per
    point, within [lo, hi]."""
    return int(min(hi, max(lo, budget_bytes // (tokens * BYTES_PER_TOKEN))))


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference", "both"], default="ours")
    ap.add_argument("--tokens", type=int, nargs="+", default=DEFAULT_TOKENS)
    ap.add_argument("--modes", nargs="+", default=list(MODES), choices=list(MODES))
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--max-reference-tokens", type=int, default=16384)
    ap.add_argument("--codec", default="none", choices=["none", "rans"],
                    help="this framework's codec (none: the reference's runnable stage set)")
    ap.add_argument("--out", default=None, help="markdown table (rank 0)")
    return ap.parse_args(argv)


def point_args(bench, world: int, tokens: int, mode: str, warmup: int,
               codec: str = "none"):
    comp, hr = MODES[mode]
    argv = ["--gpus", str(world), "--steps", str(steps_for(tokens)), "--warmup", str(warmup),
            "--tokens", str(tokens), "--requests-per-step", "1", "--compression", comp, "--no-e2e",
            "--no-full-path", "--codec", codec, "--latency-reps", "0"]
    if hr is not None:
        argv += ["--hybrid-ratio", str(hr)]
    a = bench.parse_args(argv)
    a.tag = f"{tokens}-{mode}-"
    return a


def main(argv=None) -> int:
    opts = parse_args(argv)
    import torch
    import bench
    rank, world, local = bench.dist_info()
    if world != opts.gpus:
        raise SystemExit(f"--gpus {opts.gpus} but WORLD_SIZE={world}")
    bench.init_dist(world, local)
    impls = ["ours", "reference"] if opts.impl == "both" else [opts.impl]
    rows = []
    for tokens in opts.tokens:
        for mode in opts.modes:
            for impl in impls:
                if impl == "reference" and tokens > opts.max_reference_tokens:
                    continue
                a = point_args(bench, world, tokens, mode, opts.warmup, opts.codec)
                res = bench.run_reference(a, rank, world, local) if impl == "reference" else \
                    bench.run_ours(a, rank, world, local)
                torch.cuda.empty_cache()
                if "unavailable" in res:
                    row = {"impl": impl, "unavailable": res["unavailable"]}
                else:
                    ms = res["ms"] / a.steps  # per pair: every pair hands off one request a step
                    raw = tokens * BYTES_PER_TOKEN
                    err = res.get("error") or {}
                    row = {"impl": impl, "n_gpus": world, "tokens": tokens, "raw_bytes": raw,
                           "mode": mode, "steps": a.steps, "ms_per_request": round(ms, 4),
                           "raw_gbps": round(raw / ms / 1e6, 1),
                           "compression_ratio": round(res["cr"], 3) if res.get("cr") else None,
                           "cosine": err.get("cosine"), "exact": err.get("exact"),
                           "device_error": res.get("device_error", 0),
                           "fallback_raw": res.get("fallback_raw", 0),
                           "clocks": res.get("clocks")}
                rows.append(row)
                if rank == 0:
                    print(json.dumps(row), flush=True)
    if rank == 0 and opts.out:
        with open(opts.out, "w") as f:
            f.write(render(rows))
    if world > 1:
        import torch.distributed as dist
        bench.barrier(world)
        dist.destroy_process_group()
    return 0


def render(rows) -> str:
    """Markdown table: one line per (size, mode), ours next to the reference."""
    by = {}
    for r in rows:
        if "unavailable" in r:
            continue
        by.setdefault((r["tokens"], r["mode"]), {})[r["impl"]] = r
    out = ["| raw MB/request | mode | ours ms | ours GB/s | CR | ref ms | ref GB/s | ref CR | "
           "speed-up |", "|---|---|---|---|---|---|---|---|---|"]
    for (tokens, mode), d in sorted(by.items(), key=lambda kv: (kv[0][0], list(MODES).index(kv[0][1]))):
        o, r = d.get("ours"), d.get("reference")

        def f(x, k):
            return "" if x is None or x.get(k) is None else str(x[k])
        sp = f"{r['ms_per_request'] / o['ms_per_request']:.1f}x" if o and r else ""
        if r and r.get("fallback_raw"):
            sp += " (ref sent raw: its adapter returned None)"
        out.append(f"| {tokens * BYTES_PER_TOKEN / 1e6:.1f} | {mode} | {f(o, 'ms_per_request')} | "
                   f"{f(o, 'raw_gbps')} | {f(o, 'compression_ratio')} | {f(r, 'ms_per_request')} | "
                   f"{f(r, 'raw_gbps')} | {f(r, 'compression_ratio')} | {sp} |")
    return "\n".join(out) + "\n"


if __name__ == "__main__":
    sys.exit(main())
