"""Offline profile search driver.

``python -m kvserve_hpdps_b200.offline.search --model Qwen2.5-7B-Instruct
--tolerance 3 --out results/`` evaluates candidates on synthetic (or saved)
KV with the fused kernels, runs the constraint-aware BO for the best
compression within the accuracy tolerance, and writes

* ``tolerance_<t>_results.json``: threshold, evaluations, best, history
  (the reference's result file, test_search.py:586-601);
* ``cr_cache.csv``: one row per evaluated candidate (resumable: rows already
  present are not re-evaluated);
* ``profile_library.json``: every evaluated candidate exported as a
  controller profile library.
"""

from __future__ import annotations

import argparse
import csv
import json
import os
import sys
from typing import Optional

import torch

from kvserve_hpdps_b200.offline.bo import ConstraintAwareBO, save_results
from kvserve_hpdps_b200.offline.evaluators import KVEvaluator
from kvserve_hpdps_b200.offline.library_export import build_library, write_library
from kvserve_hpdps_b200.offline.search_space import Candidate, enumerate_space

CACHE_FIELDS = ["candidate", "compression_ratio", "accuracy", "rel_mse", "cosine",
                "encode_mbps", "decode_mbps", "harmonic_speed_mbps"]


def load_cache(path: str) -> dict[str, dict]:
    if not os.path.exists(path):
        return {}
    out = {}
    with open(path) as f:
        for row in csv.DictReader(f):
            out[row["candidate"]] = {k: (float(v) if v not in ("", "None") else None)
                                     for k, v in row.items() if k != "candidate"}
    return out


def append_cache(path: str, key: str, res: dict) -> None:
    new = not os.path.exists(path)
    with open(path, "a", newline="") as f:
        w = csv.DictWriter(f, fieldnames=CACHE_FIELDS)
        if new:
            w.writeheader()
        w.writerow({"candidate": key, **{k: res.get(k) for k in CACHE_FIELDS[1:]}})


def synthetic_kv(layers: int, tokens: int, heads: int, device) -> torch.Tensor:
    from kvserve_hpdps_b200.models.synthetic import synthetic_kv as one
    return torch.stack([one(tokens, heads, seed=l, device=device) for l in range(layers)], 0)


def run_search(kv: torch.Tensor, model_name: Optional[str], tolerance: float, out_dir: str,
               budget: int = 20, space: Optional[dict] = None, measure_speed: bool = True) -> dict:
    os.makedirs(out_dir, exist_ok=True)
    ev = KVEvaluator(kv, model_name, measure_speed=measure_speed)
    cache_path = os.path.join(out_dir, "cr_cache.csv")
    cache = load_cache(cache_path)
    baseline = 1.0  # attention fidelity of the uncompressed KV
    threshold = baseline * (1 - tolerance / 100.0)

    def evaluate(c: Candidate) -> dict:
        key = c.key()
        if key in cache:
            return dict(cache[key])
        r = ev.evaluate(c).as_dict()
        r.pop("candidate")
        r.pop("config")
        cache[key] = r
        append_cache(cache_path, key, r)
        return dict(r)

    bo = ConstraintAwareBO(enumerate_space(space), evaluate, threshold, budget=budget)
    results = bo.run()
    results["tolerance"] = tolerance
    results["model_name"] = model_name
    save_results(os.path.join(out_dir, f"tolerance_{tolerance:g}_results.json"), results)
    lib = build_library(results["history"], model_name or "unknown")
    write_library(os.path.join(out_dir, "profile_library.json"), lib)
    return results


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", default="Qwen2.5-7B-Instruct")
    ap.add_argument("--tolerance", type=float, default=3.0)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--kv", help="saved KV tensor [L, 2, tokens, H, D] (torch.save)")
    ap.add_argument("--budget", type=int, default=20)
    ap.add_argument("--out", default="search_results")
    ap.add_argument("--no-speed", action="store_true")
    args = ap.parse_args(argv)
    device = "cuda" if torch.cuda.is_available() else "cpu"
    kv = torch.load(args.kv).to(device) if args.kv else \
        synthetic_kv(args.layers, args.tokens, args.heads, device)
    res = run_search(kv, args.model, args.tolerance, args.out, args.budget,
                     measure_speed=not args.no_speed)
    print(json.dumps({"best": res["best"], "evaluations": res["evaluations"]}, indent=2))
    return 0


if __name__ == "__main__":
    sys.exit(main())
