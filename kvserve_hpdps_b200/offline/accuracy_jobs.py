"""Accuracy jobs over KV-cache methods, and the collection of their results.

The reference drives accuracy with one job script per cache method
(kvserve_v1/offline_search/evaluation/lm_eval/{default,custom,kivi,cachegen,
duoattn}_accuracy.py). Each script runs lm-eval tasks and writes a log per
job. A collector then parses those logs with regular expressions into a
per-method summary CSV (lm_eval/results/collect_results.py: model, task,
configuration, score x100, compression ratio). The component-speed scripts
have their own collector (component_speed/results/collect_results.py).

Here one runner covers every method. A job is (task, method, cache
parameters) on one model. The task is either

* ``lm_eval:<task>``: an lm-eval task run through the model class that
  ``lm_harness.register_lm_eval`` adds, when lm-eval is installed; or
* a local task file (answers or choices per document, :mod:`offline.tasks`):
  the task's score x100 with the method's cache; or
* a prompt set scored by ``lm_harness.evaluate_method``: greedy-token
  agreement with the default cache (x100), first-step top-1 agreement and
  KL, and the cache's own compression ratio.  ``synthetic`` draws seeded
  random token ids; a path names a JSON list of token-id lists or a JSONL
  file with an ``input_ids`` list per row.

Every finished job appends one JSON line, so no log is parsed.  A job whose
key is already in the results file is skipped, so an interrupted sweep
resumes.  :func:`collect` keeps the newest row per key and adds the accuracy
relative to the ``default`` method of the same model and task.
:func:`collect_speed` turns ``component_speed`` output into rows of the same
kind.

    python -m kvserve_hpdps_b200.offline.accuracy_jobs run --arch Qwen2.5-7B-Instruct \\
        --layers 4 --methods default,custom,kivi --tasks synthetic --out acc.jsonl
    python -m kvserve_hpdps_b200.offline.accuracy_jobs collect acc.jsonl --csv summary.csv
    python -m kvserve_hpdps_b200.offline.accuracy_jobs collect-speed speed.jsonl --csv speed.csv
"""

from __future__ import annotations

import argparse
import csv
import json
import os
import sys
import time
from dataclasses import dataclass, field
from typing import Any, Iterable, Optional, Sequence

import torch

from kvserve_hpdps_b200.offline.tasks import is_task_file

LM_EVAL_PREFIX = "lm_eval:"


@dataclass
class Job:
    task: str
    method: str
    params: dict = field(default_factory=dict)

    def key(self, model_name: str) -> str:
        return json.dumps([model_name, self.task, self.method, self.params], sort_keys=True,
                          default=str)


def expand_jobs(methods: Sequence[str], tasks: Sequence[str],
                grid: Optional[dict[str, list[dict]]] = None) -> list[Job]:
    """Every (task, method, parameter set): a method's parameter sets come
    from ``grid`` (each merged over the method's defaults), else its
    defaults alone (``cr_methods.DEFAULT_PARAMS``)."""
    from kvserve_hpdps_b200.offline.cr_methods import DEFAULT_PARAMS
    jobs = []
    for t in tasks:
        for m in methods:
            sets = (grid or {}).get(m) or [{}]
            for extra in sets:
                p = dict(DEFAULT_PARAMS.get(m, {}))
                p.update(extra)
                jobs.append(Job(t, m, p))
    return jobs


def load_prompts(task: str, vocab_size: int, tokens: int = 512, count: int = 4,
                 seed: int = 0) -> list[torch.Tensor]:
    """Token-id prompts of a prompt-set task (see the module docstring)."""
    if task == "synthetic":
        g = torch.Generator().manual_seed(seed)
        return [torch.randint(0, vocab_size, (tokens,), generator=g) for _ in range(count)]
    if not os.path.exists(task):
        raise ValueError(f"unknown task {task!r}: expected 'synthetic', a prompt file, a task "
                         f"file or {LM_EVAL_PREFIX}<task>")
    with open(task) as f:
        text = f.read()
    try:
        data = json.loads(text)
        rows = data if isinstance(data, list) else [data]
    except json.JSONDecodeError:
        rows = [json.loads(line) for line in text.splitlines() if line.strip()]
    out = []
    for r in rows[:count] if count else rows:
        ids = r.get("input_ids") if isinstance(r, dict) else r
        if not isinstance(ids, list) or not ids:
            raise ValueError(f"{task}: each prompt must be a non-empty list of token ids")
        out.append(torch.tensor([int(i) for i in ids], dtype=torch.long))
    return out


def _lm_eval_job(model_name: str, job: Job, model_args: str, limit: Optional[int]) -> dict:
    """One lm-eval task with a method's cache (lm-eval installed): the score
    is the first metric of the task, x100, as the reference's collector
    reports it."""
    try:
        import lm_eval
    except ImportError as e:  # pragma: no cover - lm-eval is not in this image
        raise RuntimeError("lm-eval is not installed; use a prompt-set task") from e
    from kvserve_hpdps_b200.offline.lm_harness import register_lm_eval
    name = "my_custom_model"  # the model name the reference's job scripts pass
    register_lm_eval(name)
    args = ",".join([a for a in (model_args,) if a] + [f"cache_type={job.method}"] +
                    [f"{k}={v}" for k, v in job.params.items()])
    task = job.task[len(LM_EVAL_PREFIX):]
    res = lm_eval.simple_evaluate(model=name, model_args=args, tasks=[task], limit=limit)
    metrics = res["results"][task]
    first = next((v for k, v in metrics.items() if isinstance(v, (int, float))
                  and not k.endswith("_stderr") and "stderr" not in k), float("nan"))
    return {"accuracy": round(100.0 * float(first), 4), "backend": "lm-eval",
            "metrics": {k: v for k, v in metrics.items() if isinstance(v, (int, float))}}


def _task_file_job(model, job: Job, scores: Optional[torch.Tensor], limit: Optional[int],
                   tokenizer=None) -> dict:
    """A local task file (:mod:`offline.tasks`) with the method's cache: the
    accuracy is the task's score x100 over its first ``limit`` documents."""
    from kvserve_hpdps_b200.offline.lm_harness import CacheMethodModel
    from kvserve_hpdps_b200.offline.tasks import TaskRunner, load_task
    task = load_task(job.task)
    params = dict(job.params)
    if job.method == "custom":
        params.setdefault("device", str(model.device))
    cm = CacheMethodModel(model, job.method, scores if job.method != "default" else None,
                          **params)
    try:
        n = len(task.docs) if not limit else min(limit, len(task.docs))
        r = TaskRunner(cm, tokenizer).run(task, range(n))
        cache = cm.last_cache
        cr = float(cache.compute_compression_ratio()) \
            if hasattr(cache, "compute_compression_ratio") else 1.0
    finally:
        cm.close()
    return {"accuracy": round(100.0 * r["score"], 4), "backend": "task-file",
            "metrics": {k: v for k, v in r.items() if k != "docs"}, "docs": r["docs"],
            "compression_ratio": cr}


def run_job(model, model_name: str, job: Job, scores: Optional[torch.Tensor] = None,
            tokens: int = 512, prompts: int = 4, max_new_tokens: int = 16,
            model_args: str = "", limit: Optional[int] = None, tokenizer=None) -> dict:
    """Run one job; returns its result row."""
    from kvserve_hpdps_b200.offline.lm_harness import evaluate_method
    t0 = time.monotonic()
    row = {"model": model_name, "task": job.task, "method": job.method,
           "config": dict(job.params)}
    if job.task.startswith(LM_EVAL_PREFIX):
        row.update(_lm_eval_job(model_name, job, model_args, limit))
    elif is_task_file(job.task):
        row.update(_task_file_job(model, job, scores, limit, tokenizer))
    else:
        ps = load_prompts(job.task, int(model.config.vocab_size), tokens, prompts)
        params = dict(job.params)
        if job.method == "custom":
            params.setdefault("device", str(model.device))
        r = evaluate_method(model, ps, job.method, scores=scores,
                            max_new_tokens=max_new_tokens, **params)
        row.update({"accuracy": round(r.accuracy, 4), "top1_agreement": r.top1_agreement,
                    "kl": r.kl, "compression_ratio": r.compression_ratio,
                    "backend": "prompt-set", "prompts": len(ps),
                    "prompt_tokens": int(ps[0].numel()) if ps else 0})
    row["seconds"] = round(time.monotonic() - t0, 3)
    row["key"] = job.key(model_name)
    return row


def read_rows(path: str) -> list[dict]:
    if not os.path.exists(path):
        return []
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


def run_jobs(model, model_name: str, jobs: Iterable[Job], out_path: str,
             scores: Optional[torch.Tensor] = None, resume: bool = True,
             **kwargs: Any) -> list[dict]:
    """Run the jobs, appending each row to ``out_path`` as it finishes;
    with ``resume`` the jobs whose key is already there are skipped."""
    done = {r.get("key") for r in read_rows(out_path)} if resume else set()
    rows = []
    for job in jobs:
        if job.key(model_name) in done:
            continue
        row = run_job(model, model_name, job, scores, **kwargs)
        with open(out_path, "a") as f:
            f.write(json.dumps(row, default=str) + "\n")
        rows.append(row)
    return rows


SUMMARY_FIELDS = ("model", "task", "method", "config", "backend", "accuracy",
                  "accuracy_vs_default", "compression_ratio", "top1_agreement", "kl", "seconds")


def collect(rows: Iterable[dict]) -> list[dict]:
    """Summary rows: the newest row per job key, sorted by model, task and
    method, with ``accuracy_vs_default`` = accuracy / the ``default``
    method's accuracy on the same model and task x100 (the reference's
    search normalises task scores the same way)."""
    latest: dict[str, dict] = {}
    for r in rows:
        latest[r.get("key") or json.dumps([r.get("model"), r.get("task"), r.get("method"),
                                           r.get("config")], sort_keys=True, default=str)] = r
    base = {(r["model"], r["task"]): r.get("accuracy") for r in latest.values()
            if r.get("method") == "default"}
    out = []
    for r in latest.values():
        s = {k: r.get(k) for k in SUMMARY_FIELDS}
        s["config"] = json.dumps(r.get("config") or {}, sort_keys=True)
        b = base.get((r.get("model"), r.get("task")))
        acc = r.get("accuracy")
        s["accuracy_vs_default"] = (round(100.0 * acc / b, 2)
                                    if isinstance(acc, (int, float)) and b else None)
        out.append(s)
    order = {"default": 0}
    out.sort(key=lambda s: (str(s["model"]), str(s["task"]), order.get(s["method"], 1),
                            str(s["method"]), s["config"]))
    return out


def collect_speed(lines: Iterable[str], source: str = "") -> list[dict]:
    """Rows of ``component_speed`` output (one JSON object per line): one
    row per timed stage, with the run's compression ratio from its
    ``summary`` line; lines that are not JSON objects are skipped."""
    stages, summary = [], {}
    for line in lines:
        line = line.strip()
        if not line.startswith("{"):
            continue
        try:
            r = json.loads(line)
        except json.JSONDecodeError:
            continue
        if r.get("stage") == "summary":
            summary = r
        elif "stage" in r:
            stages.append(r)
    out = []
    for r in stages:
        out.append({"source": source, "stage": r["stage"], "ms": r.get("ms"),
                    "gbps": r.get("gbps"), "layers": r.get("layers"),
                    "tokens": r.get("tokens"), "heads": r.get("heads"),
                    "code_width": summary.get("code_width"),
                    "compression_ratio": summary.get("compression_ratio")})
    return out


def write_csv(rows: Sequence[dict], path: Optional[str]) -> None:
    if not rows:
        return
    f = open(path, "w", newline="") if path else sys.stdout
    try:
        w = csv.DictWriter(f, fieldnames=list(rows[0]))
        w.writeheader()
        w.writerows(rows)
    finally:
        if path:
            f.close()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run", help="run accuracy jobs, appending rows to --out")
    r.add_argument("--arch", default="Qwen2.5-7B-Instruct",
                   help="random-init architecture (no checkpoint needed)")
    r.add_argument("--model", default=None, help="local Hugging Face checkpoint directory")
    r.add_argument("--layers", type=int, default=None)
    r.add_argument("--hidden", type=int, default=None)
    r.add_argument("--methods", default="default,custom,kivi,cachegen,duoattn")
    r.add_argument("--tasks", default="synthetic",
                   help="comma list: synthetic | prompt file | lm_eval:<task>")
    r.add_argument("--grid", default=None,
                   help="JSON {method: [parameter sets]} swept per method")
    r.add_argument("--tokens", type=int, default=512)
    r.add_argument("--prompts", type=int, default=4)
    r.add_argument("--new-tokens", type=int, default=16)
    r.add_argument("--limit", type=int, default=None,
                   help="documents per task (lm-eval tasks and task files)")
    r.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    r.add_argument("--out", required=True)
    r.add_argument("--no-resume", action="store_true")
    c = sub.add_parser("collect", help="summarise result rows into a CSV")
    c.add_argument("results", nargs="+")
    c.add_argument("--csv", default=None)
    sp = sub.add_parser("collect-speed", help="component_speed output files into a CSV")
    sp.add_argument("inputs", nargs="+")
    sp.add_argument("--csv", default=None)
    args = ap.parse_args(argv)

    if args.cmd == "collect":
        rows = [row for p in args.results for row in read_rows(p)]
        write_csv(collect(rows), args.csv)
        return 0
    if args.cmd == "collect-speed":
        out = []
        for p in args.inputs:
            with open(p) as f:
                out += collect_speed(f, source=os.path.basename(p))
        write_csv(out, args.csv)
        return 0

    from kvserve_hpdps_b200.compression.head_scores import get_scores_from_csv, synthetic_scores
    from kvserve_hpdps_b200.offline.cr_methods import random_model
    dtype = torch.bfloat16 if args.device.startswith("cuda") else torch.float32
    model_args = ""
    tokenizer = None
    if args.model:
        from transformers import AutoModelForCausalLM, AutoTokenizer
        model = AutoModelForCausalLM.from_pretrained(args.model, torch_dtype=dtype).to(args.device)
        name = os.path.basename(os.path.normpath(args.model))
        model_args = f"pretrained={args.model}"
        try:  # text task files need it; id-only tasks and prompt sets do not
            tokenizer = AutoTokenizer.from_pretrained(args.model, local_files_only=True)
        except (OSError, ValueError):
            tokenizer = None
    else:
        model, spec = random_model(args.arch, args.layers, args.hidden, dtype=dtype,
                                   device=args.device)
        name = spec.name
    L, H = model.config.num_hidden_layers, model.config.num_key_value_heads
    scores = get_scores_from_csv(name)
    if scores is None or tuple(scores.shape) != (L, H):
        scores = synthetic_scores(L, H)
    jobs = expand_jobs(args.methods.split(","), args.tasks.split(","),
                       json.loads(args.grid) if args.grid else None)
    rows = run_jobs(model, name, jobs, args.out, scores, resume=not args.no_resume,
                    tokens=args.tokens, prompts=args.prompts, max_new_tokens=args.new_tokens,
                    model_args=model_args, limit=args.limit, tokenizer=tokenizer)
    print(json.dumps({"jobs": len(jobs), "ran": len(rows), "out": args.out}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
