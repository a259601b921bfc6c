"""Model-based evaluators of the offline parameter search: compression ratio
and task accuracy of a custom-cache configuration on a causal LM.

These keep the interface of the reference's evaluators
(kvserve_v1/offline_search/evaluation/param_search/cr_evaluator.py:19-173 and
acc_evaluator.py:68-242): constructed once per search with the model name,
the tasks, the document limit and the seed; ``evaluate(params)`` takes a
search-space point (``transform_type``, ``heads_selection``, the four max
values, ``axis_key``, ``axis_value``) and returns a number.

* :class:`CompressionEvaluator` prefills the longest document of a task (or
  a given prompt) through the custom cache and returns original bf16 bytes
  over coded bytes (codes through this package's rANS coder + metadata),
  rounded to 4 places.
* :class:`AccuracyEvaluator` scores the tasks once with the default cache,
  then per configuration with the custom cache, and returns the mean of
  (custom / default) over the tasks x100, rounded to 2 places.  Tasks are
  local task files (:mod:`offline.tasks`), or lm-eval task names when
  lm-eval is installed (run through the model class of
  ``lm_harness.register_lm_eval`` with the same document sample).

Documents are sampled as the reference samples them: with ``limit`` below a
task's size, one document from each of ``limit`` equal intervals, drawn by
one ``random.Random(random_seed)`` shared by the tasks in order, so a search
here and the reference's search on the same task evaluate the same
documents.

Without a local checkpoint (``base_model_path/model_name``) the model is a
random-init network of the named architecture; head scores come from
``base_config_path/<model>_scores.csv`` or the package's tables.
"""

from __future__ import annotations

import os
import random
from typing import Any, Optional, Sequence

import torch

from kvserve_hpdps_b200.offline.tasks import LocalTask, TaskRunner, is_task_file, load_task

# Whether lm-eval should wrap a task's prompt in the model's chat template
# (the reference's table, acc_evaluator.py:20-42): instruction-following QA
# and summarisation tasks yes; code completion and classification no.
TASK_TO_CHAT_TEMPLATE = {
    "longbench_lcc": False, "longbench_lcc_e": False,
    "longbench_repobench-p": False, "longbench_repobench-p_e": False,
    "longbench_multi_news": True, "longbench_multi_news_e": True,
    "longbench_gov_report": True, "longbench_gov_report_e": True,
    "longbench_2wikimqa": True, "longbench_2wikimqa_e": True,
    "longbench_hotpotqa": True, "longbench_hotpotqa_e": True,
    "longbench_qasper": True, "longbench_qasper_e": True,
    "longbench_multifieldqa_en": True, "longbench_multifieldqa_en_e": True,
    "longbench_trec": False,
    "gsm8k_cot_llama": True, "gsm8k_cot": False,
    "mbpp_instruct": True, "humaneval_instruct": True,
}

PARAM_KEYS = ("transform_type", "heads_selection", "high_key_max_value", "high_value_max_value",
              "low_key_max_value", "low_value_max_value", "axis_key", "axis_value")


def stratified_indices(n_docs: int, limit: int, rng: random.Random) -> list[int]:
    """All documents when ``n_docs <= limit``; else one index drawn from each
    of ``limit`` evenly spaced intervals of ``[0, n_docs)``."""
    if n_docs <= limit:
        return list(range(n_docs))
    step = n_docs / limit
    out = []
    for i in range(limit):
        lo = int(i * step)
        hi = min(max(int((i + 1) * step), lo + 1), n_docs)
        out.append(rng.randrange(lo, hi) if lo < hi else lo)
    return out


def load_model(model_name: str, base_model_path: Optional[str] = None, device: str = "cpu",
               dtype=None, layers: Optional[int] = None, hidden: Optional[int] = None,
               seed: int = 0):
    """(model, tokenizer): a local checkpoint at ``base_model_path/model_name``
    when it exists (no network), else a random-init model of the named
    architecture (optionally shrunk) and no tokenizer."""
    path = os.path.join(base_model_path, model_name) if base_model_path else None
    if path and os.path.isdir(path):
        from transformers import AutoModelForCausalLM, AutoTokenizer
        model = AutoModelForCausalLM.from_pretrained(path, torch_dtype=dtype or "auto",
                                                     local_files_only=True)
        try:
            tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        except (OSError, ValueError):
            tok = None
        return model.to(device).eval(), tok
    from kvserve_hpdps_b200.offline.cr_methods import random_model
    model, _ = random_model(model_name, layers=layers, hidden=hidden, seed=seed,
                            dtype=dtype or torch.float32, device=device)
    return model, None


def load_scores(model_name: str, base_config_path: Optional[str], num_layers: int,
                num_heads: int) -> torch.Tensor:
    """[layers, kv_heads] head scores: ``base_config_path/<model>_scores.csv``,
    else the package's table, else the deterministic synthetic table.  A
    table of another shape (a shrunk test model) is cut or tiled to fit."""
    from kvserve_hpdps_b200.compression.head_scores import (_read_csv, get_scores_from_csv,
                                                            synthetic_scores)
    t = None
    if base_config_path:
        p = os.path.join(base_config_path, f"{model_name}_scores.csv")
        if os.path.exists(p):
            t = _read_csv(p)
    if t is None:
        t = get_scores_from_csv(model_name)
    if t is None:
        return synthetic_scores(num_layers, num_heads)
    if tuple(t.shape) != (num_layers, num_heads):
        t = t.repeat((num_layers + t.shape[0] - 1) // t.shape[0],
                     (num_heads + t.shape[1] - 1) // t.shape[1])[:num_layers, :num_heads]
    return t.contiguous()


def custom_params(params: dict, device) -> dict:
    """A search-space point as ``CustomCacheConfig`` fields."""
    missing = [k for k in PARAM_KEYS if k not in params]
    if missing:
        raise ValueError(f"search parameters without {missing}")
    out = {k: params[k] for k in PARAM_KEYS}
    out["axis_key"] = list(out["axis_key"])
    out["axis_value"] = list(out["axis_value"])
    out["device"] = str(device)
    return out


def candidate_params(c) -> dict:
    """An :class:`offline.search_space.Candidate` as a search-space point of
    the reference's form (Hadamard transform; ``channel`` keys reduce over
    tokens, ``token`` values over heads and head_dim)."""
    axes = {"channel": [2], "token": [1, 3], "tensor": [1, 2, 3]}
    return {"transform_type": "hadamard", "heads_selection": float(c.hybrid_ratio),
            "high_key_max_value": int(c.high_key_max_value),
            "high_value_max_value": int(c.high_value_max_value),
            "low_key_max_value": int(c.low_key_max_value),
            "low_value_max_value": int(c.low_value_max_value),
            "axis_key": axes[c.axis_key], "axis_value": axes[c.axis_value]}


def _resolve_task(name: str, task_dirs: Sequence[str]) -> Optional[str]:
    if is_task_file(name):
        return name
    for d in task_dirs:
        for ext in (".json", ".jsonl"):
            p = os.path.join(d, name + ext)
            if is_task_file(p):
                return p
    return None


class _ModelHolder:
    def __init__(self, model_name, base_model_path, base_config_path, device, model, tokenizer,
                 scores, model_kwargs):
        self.model_name = model_name
        self.base_model_path = base_model_path
        self.base_config_path = base_config_path
        if model is None:
            model, tok = load_model(model_name, base_model_path, device, **(model_kwargs or {}))
            tokenizer = tokenizer if tokenizer is not None else tok
        self.model = model.eval()
        self.tokenizer = tokenizer
        cfg = self.model.config
        self.num_layers = int(cfg.num_hidden_layers)
        self.num_kv_heads = int(getattr(cfg, "num_key_value_heads", None)
                                or cfg.num_attention_heads)
        self.scores = scores if scores is not None else \
            load_scores(model_name, base_config_path, self.num_layers, self.num_kv_heads)

    def cache_model(self, method: str, **params: Any):
        from kvserve_hpdps_b200.offline.lm_harness import CacheMethodModel
        return CacheMethodModel(self.model, method, self.scores if method != "default" else None,
                                **params)


class CompressionEvaluator(_ModelHolder):
    """Compression ratio of a configuration on one long input."""

    def __init__(self, model_name: str = "Qwen2.5-7B-Instruct", task: Optional[str] = None,
                 device: str = "cpu", base_model_path: Optional[str] = None,
                 base_config_path: Optional[str] = None, *, model=None, tokenizer=None,
                 scores: Optional[torch.Tensor] = None, input_ids: Optional[torch.Tensor] = None,
                 task_dirs: Sequence[str] = (), synthetic_tokens: int = 2048,
                 model_kwargs: Optional[dict] = None):
        super().__init__(model_name, base_model_path, base_config_path, device, model, tokenizer,
                         scores, model_kwargs)
        if input_ids is None and task:
            path = _resolve_task(task, task_dirs)
            if path is None:
                raise ValueError(f"no local task file for {task!r}")
            input_ids = self._longest_context(load_task(path))
        if input_ids is None:  # a seeded synthetic prompt of the requested length
            g = torch.Generator().manual_seed(0)
            input_ids = torch.randint(0, int(self.model.config.vocab_size), (synthetic_tokens,),
                                      generator=g)
        self.input_ids = input_ids.view(1, -1).to(self.model.device)

    def _longest_context(self, task: LocalTask) -> torch.Tensor:
        runner = TaskRunner(None, self.tokenizer)
        ids = [runner._ids(d, "context", task) for d in task.docs]
        return torch.tensor(max(ids, key=len), dtype=torch.long)

    @torch.no_grad()
    def evaluate(self, params: dict) -> float:
        from kvserve_hpdps_b200.offline import caches as C
        cfg = C.CustomCacheConfig(scores=self.scores, **custom_params(params, self.model.device))
        cache = C.CustomCache(cfg)
        self.model(self.input_ids, past_key_values=cache, use_cache=True)  # prefill only
        return float(cache.compute_compression_ratio())


class AccuracyEvaluator(_ModelHolder):
    """Task accuracy of a configuration relative to the default cache (x100)."""

    def __init__(self, model_name: str = "Meta-Llama-3.1-8B-Instruct",
                 tasks: Sequence[str] = ("longbench_hotpotqa",), limit: int = 100,
                 batch_size: int = 1, device: str = "cpu", random_seed: int = 42,
                 base_model_path: Optional[str] = None, base_config_path: Optional[str] = None,
                 *, model=None, tokenizer=None, scores: Optional[torch.Tensor] = None,
                 task_dirs: Sequence[str] = (), task_overrides: Optional[dict] = None,
                 model_kwargs: Optional[dict] = None):
        super().__init__(model_name, base_model_path, base_config_path, device, model, tokenizer,
                         scores, model_kwargs)
        self.tasks = list(tasks)
        self.limit = int(limit)
        self.batch_size = int(batch_size)
        self.random_seed = random_seed
        self.local: dict[str, LocalTask] = {}
        self.lm_eval_tasks: list[str] = []
        for t in self.tasks:
            p = _resolve_task(t, task_dirs)
            if p is not None:
                self.local[t] = load_task(p, **(task_overrides or {}))
            else:
                self.lm_eval_tasks.append(t)
        self.samples = self._sample()
        self.default_scores = self._scores("default", {})

    def _lm_eval_docs(self) -> dict[str, int]:
        try:
            from lm_eval.tasks import TaskManager, get_task_dict
        except ImportError as e:
            raise RuntimeError(
                f"tasks {self.lm_eval_tasks} are neither local task files nor runnable: "
                "lm-eval is not installed") from e
        out = {}
        for name, task in get_task_dict(self.lm_eval_tasks, TaskManager()).items():
            if getattr(task, "has_test_docs", lambda: False)():
                docs = task.test_docs()
            elif getattr(task, "has_validation_docs", lambda: False)():
                docs = task.validation_docs()
            else:
                docs = task.training_docs()
            out[name] = len(docs) if hasattr(docs, "__len__") else len(list(docs))
        return out

    def _sample(self) -> dict[str, list[int]]:
        """Document indices per task: local tasks in the order given, then
        lm-eval tasks in lm-eval's order, one seeded generator for all."""
        rng = random.Random(self.random_seed)
        sizes = {name: len(self.local[name].docs) for name in self.tasks if name in self.local}
        if self.lm_eval_tasks:
            sizes.update(self._lm_eval_docs())
        return {name: stratified_indices(n, self.limit, rng) for name, n in sizes.items()}

    def _scores(self, method: str, params: dict) -> list[float]:
        """One ``score`` per task, in task order (local tasks, then lm-eval)."""
        out = []
        cm = self.cache_model(method, **params)
        try:
            runner = TaskRunner(cm, self.tokenizer)
            for name in self.tasks:
                if name in self.local:
                    out.append(round(runner.run(self.local[name], self.samples[name])["score"], 4))
        finally:
            cm.close()
        if self.lm_eval_tasks:
            out.extend(self._lm_eval_scores(method, params))
        return out

    def _lm_eval_scores(self, method: str, params: dict) -> list[float]:  # pragma: no cover
        import lm_eval

        from kvserve_hpdps_b200.offline.lm_harness import register_lm_eval
        register_lm_eval("my_custom_model")
        args = {"pretrained": os.path.join(self.base_model_path or "", self.model_name),
                "cache_type": method, **params}
        if method != "default":
            args["scores"] = self.scores
        vals = []
        for task in self.lm_eval_tasks:
            res = lm_eval.simple_evaluate(
                model="my_custom_model", model_args=args, tasks=[task],
                batch_size=self.batch_size,
                apply_chat_template=TASK_TO_CHAT_TEMPLATE.get(task, False),
                confirm_run_unsafe_code=True,
                samples={k: v for k, v in self.samples.items() if k not in self.local})
            for metrics in res["results"].values():
                vals.extend(round(float(v), 4) for k, v in metrics.items()
                            if "score" in k and "_stderr" not in k)
        return vals

    def evaluate(self, params: dict) -> float:
        """Mean over the tasks of custom score / default score, x100.  A task
        that the default cache scores 0 gives no ratio and is left out (all
        left out: 100.0)."""
        got = self._scores("custom", custom_params(params, self.model.device))
        ratios = [c / d for c, d in zip(got, self.default_scores) if d > 0]
        if not ratios:
            return 100.0
        return round(100.0 * sum(ratios) / len(ratios), 2)
