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

With ``--tasks`` the search runs on a causal LM instead, as the reference's
driver does: compression ratio from a prefill through the custom cache and
accuracy as task score relative to the default cache (x100, threshold
100 - tolerance), from local task files or lm-eval tasks
(:mod:`offline.param_search`).  The model is a checkpoint under
``--base-model-path`` or a random-init network of the named architecture.
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
    """Search on a KV stack: accuracy is the attention fidelity of the
    reconstructed KV (1.0 = exact), the threshold 1 - tolerance/100."""
    ev = KVEvaluator(kv, model_name, measure_speed=measure_speed)

    def evaluate(c: Candidate) -> dict:
        r = ev.evaluate(c).as_dict()
        r.pop("candidate")
        r.pop("config")
        return r

    return _search(evaluate, 1.0 * (1 - tolerance / 100.0), model_name, tolerance, out_dir,
                   budget, space, signature={"mode": "kv", "model": model_name,
                                             "kv_shape": list(kv.shape)})


def run_model_search(model_name: str, tasks: list[str], tolerance: float, out_dir: str,
                     budget: int = 20, space: Optional[dict] = None, limit: int = 5,
                     seed: int = 42, base_model_path: Optional[str] = None,
                     base_config_path: Optional[str] = None, task_dirs: tuple = (),
                     device: str = "cpu", cr_task: Optional[str] = None,
                     model=None, tokenizer=None, model_kwargs: Optional[dict] = None) -> dict:
    """Search on a causal LM as the reference's driver does: compression
    ratio from a prefill through the custom cache, accuracy = task score
    relative to the default cache x100, threshold 100 - tolerance
    (kvserve_v1/offline_search/evaluation/param_search/test_search.py:24-27)."""
    from kvserve_hpdps_b200.offline.param_search import (AccuracyEvaluator, CompressionEvaluator,
                                                         candidate_params)
    acc = AccuracyEvaluator(model_name, tasks, limit=limit, device=device, random_seed=seed,
                            base_model_path=base_model_path, base_config_path=base_config_path,
                            model=model, tokenizer=tokenizer, task_dirs=task_dirs,
                            model_kwargs=model_kwargs)
    cr = CompressionEvaluator(model_name, cr_task or tasks[0], device, base_model_path,
                              base_config_path, model=acc.model, tokenizer=acc.tokenizer,
                              scores=acc.scores, task_dirs=task_dirs)
    speed = None
    if torch.cuda.is_available():
        # the controller needs each profile's compress/decompress speed: timed
        # with the fused kernels on synthetic KV of the model's per-rank shape
        heads = int(getattr(acc.model.config, "num_key_value_heads", 0) or
                    acc.model.config.num_attention_heads)
        speed = KVEvaluator(synthetic_kv(4, 2048, heads, "cuda"), model_name)
    else:
        print("search: no GPU, profile speeds are not measured (the library gets a "
              "placeholder of 1e6 MB/s)", file=sys.stderr)

    def evaluate(c: Candidate) -> dict:
        p = candidate_params(c)
        out = {"compression_ratio": cr.evaluate(p), "accuracy": acc.evaluate(p)}
        if speed is not None:
            r = speed.evaluate(c)
            out.update(encode_mbps=r.encode_mbps, decode_mbps=r.decode_mbps,
                       harmonic_speed_mbps=r.harmonic_speed_mbps)
        return out

    # task accuracy is x100 of the default cache's; library accuracy is a fraction
    res = _search(evaluate, 100.0 - tolerance, model_name, tolerance, out_dir, budget, space,
                  library_acc_scale=0.01,
                  signature={"mode": "tasks", "model": model_name, "tasks": list(tasks),
                             "limit": int(limit), "seed": int(seed)})
    res["tasks"] = list(tasks)
    res["default_scores"] = list(acc.default_scores)
    save_results(os.path.join(out_dir, f"tolerance_{tolerance:g}_results.json"), res)
    return res


def check_signature(out_dir: str, signature: Optional[dict]) -> None:
    """The evaluation cache of ``out_dir`` belongs to one search (mode, model,
    KV shape or tasks, sample): ``search_signature.json`` records it, and a
    search with another signature refuses to resume from that cache."""
    if signature is None:
        return
    path = os.path.join(out_dir, "search_signature.json")
    if os.path.exists(path):
        with open(path) as f:
            old = json.load(f)
        if old != json.loads(json.dumps(signature)):
            raise ValueError(f"{out_dir} holds the cache of another search ({old}); use a new "
                             f"output directory for {signature}")
        return
    with open(path, "w") as f:
        json.dump(signature, f, indent=2)


def _search(evaluate_fn, threshold: float, model_name: Optional[str], tolerance: float,
            out_dir: str, budget: int, space: Optional[dict],
            library_acc_scale: float = 1.0, signature: Optional[dict] = None) -> dict:
    os.makedirs(out_dir, exist_ok=True)
    check_signature(out_dir, signature)
    cache_path = os.path.join(out_dir, "cr_cache.csv")
    cache = load_cache(cache_path)

    def evaluate(c: Candidate) -> dict:
        key = c.key()
        if key in cache:
            return dict(cache[key])
        r = evaluate_fn(c)
        cache[key] = r
        append_cache(cache_path, key, r)
        return dict(r)

    bo = ConstraintAwareBO(enumerate_space(space), evaluate, threshold, budget=budget)
    results = bo.run()
    results["tolerance"] = tolerance
    results["model_name"] = model_name
    save_results(os.path.join(out_dir, f"tolerance_{tolerance:g}_results.json"), results)
    hist = [dict(h, accuracy=h["accuracy"] * library_acc_scale) for h in results["history"]]
    lib = build_library(hist, model_name or "unknown")
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
    ap.add_argument("--tasks", help="comma-separated tasks: search on a model with task accuracy "
                    "(local task files, or lm-eval task names when lm-eval is installed)")
    ap.add_argument("--task-dir", action="append", default=[],
                    help="directory holding <task>.json / <task>.jsonl files")
    ap.add_argument("--limit", type=int, default=5, help="documents per task")
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--base-model-path", help="directory holding <model>/ checkpoints")
    ap.add_argument("--base-config-path", help="directory holding <model>_scores.csv")
    ap.add_argument("--model-layers", type=int, help="random-init model: number of layers")
    args = ap.parse_args(argv)
    device = "cuda" if torch.cuda.is_available() else "cpu"
    if args.tasks:
        res = run_model_search(args.model, args.tasks.split(","), args.tolerance, args.out,
                               args.budget, limit=args.limit, seed=args.seed,
                               base_model_path=args.base_model_path,
                               base_config_path=args.base_config_path,
                               task_dirs=tuple(args.task_dir), device=device,
                               model_kwargs={"layers": args.model_layers})
        print(json.dumps({"best": res["best"], "evaluations": res["evaluations"]}, indent=2))
        return 0
    print(json.dumps({"best": res["best"], "evaluations": res["evaluations"]}, indent=2))
    return 0


if __name__ == "__main__":
    sys.exit(main())
