"""Task accuracy of KV-cache methods on local task files, without lm-eval.

The reference scores a cache configuration with lm-eval tasks, mostly
LongBench generation tasks whose metric is a token F1 against reference
answers, on a fixed sample of documents
(kvserve_v1/offline_search/evaluation/param_search/acc_evaluator.py:68-242,
lm_eval/lm_wrapper.py:157-219).  lm-eval and its datasets are not reachable
offline, so this module runs the same kind of evaluation on task files that
a user places on disk, through the same cache methods
(:class:`lm_harness.CacheMethodModel`).

Task file: JSON (``{"name", "kind", "metric", "max_new_tokens",
"chat_template", "docs": [...]}``) or JSONL (one document per line; the
settings then come from the defaults or the caller).  Documents carry text
(tokenized with the model's tokenizer) or token ids:

* ``kind: "generate"``: ``context`` / ``context_ids``, ``answers`` (list of
  strings) / ``answers_ids`` (list of id lists), optional ``stop`` /
  ``stop_ids``.  Greedy generation with the method's cache; metrics
  ``qa_f1`` (token F1 after answer normalisation, best over answers),
  ``exact_match`` and ``contains`` (an answer appears in the output).
* ``kind: "choice"``: ``context`` / ``context_ids``, ``choices`` /
  ``choices_ids``, ``gold`` (index).  Each continuation is scored by its
  log-likelihood after a prefill of the context into the method's cache, so
  the continuation attends to the reconstructed KV (lm-eval scores a
  continuation in one forward with the context, where a compressed cache
  would never be read); metric ``acc``.

The kind defaults to ``choice`` when the first document has choices, else
``generate``.  A task's ``score`` is its primary metric (``qa_f1`` or
``acc``); the reference's evaluator likewise normalises the metric named
``score``.

Answer normalisation and token F1 follow the SQuAD v1.1 evaluation
(Rajpurkar et al., 2016: lower case, drop punctuation and the articles
a/an/the, collapse white space; F1 over the multiset of tokens), the form
LongBench's QA metric uses.  Id-only documents use the same F1 over token
ids.
"""

from __future__ import annotations

import json
import os
import re
import string
from collections import Counter
from dataclasses import dataclass, field
from typing import Any, Optional, Sequence

import torch

KINDS = ("generate", "choice")
PRIMARY_METRIC = {"generate": "qa_f1", "choice": "acc"}


@dataclass
class LocalTask:
    name: str
    kind: str
    docs: list
    metric: Optional[str] = None
    max_new_tokens: int = 32
    chat_template: bool = False
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        if self.kind not in KINDS:
            raise ValueError(f"task {self.name!r}: kind must be one of {KINDS}, got {self.kind!r}")
        if not self.docs:
            raise ValueError(f"task {self.name!r} has no documents")
        self.metric = self.metric or PRIMARY_METRIC[self.kind]


def is_task_file(path: str) -> bool:
    """True for a JSON/JSONL file whose documents look like task documents
    (answers or choices), as opposed to a bare prompt set."""
    if not isinstance(path, str) or not os.path.isfile(path):
        return False
    try:
        obj = _read_json_or_jsonl(path)
    except (OSError, ValueError):
        return False
    docs = obj.get("docs") if isinstance(obj, dict) else obj
    if isinstance(obj, dict) and "kind" in obj:
        return True
    first = docs[0] if isinstance(docs, list) and docs else None
    return isinstance(first, dict) and any(
        k in first for k in ("answers", "answers_ids", "choices", "choices_ids"))


def _read_json_or_jsonl(path: str):
    with open(path) as f:
        text = f.read()
    try:
        return json.loads(text)
    except json.JSONDecodeError:
        return [json.loads(line) for line in text.splitlines() if line.strip()]


def load_task(path: str, **overrides: Any) -> LocalTask:
    """Read a task file (see the module docstring); ``overrides`` replace the
    file's settings (``max_new_tokens=...`` and the like)."""
    obj = _read_json_or_jsonl(path)
    if isinstance(obj, dict):
        settings = {k: v for k, v in obj.items() if k != "docs"}
        docs = obj.get("docs") or []
    else:
        settings, docs = {}, obj
    settings.update(overrides)
    name = settings.pop("name", None) or os.path.splitext(os.path.basename(path))[0]
    kind = settings.pop("kind", None)
    if kind is None:
        first = docs[0] if docs else {}
        kind = "choice" if ("choices" in first or "choices_ids" in first) else "generate"
    known = {"metric", "max_new_tokens", "chat_template"}
    extra = {k: settings.pop(k) for k in list(settings) if k not in known}
    return LocalTask(name=name, kind=kind, docs=list(docs), extra=extra, **settings)


# ---------------------------------------------------------------- metrics

_ARTICLES = re.compile(r"\b(a|an|the)\b")
_PUNCT = set(string.punctuation)


def normalize_answer(s: str) -> str:
    s = s.lower()
    s = "".join(ch for ch in s if ch not in _PUNCT)
    s = _ARTICLES.sub(" ", s)
    return " ".join(s.split())


def token_f1(pred: Sequence, gold: Sequence) -> float:
    common = Counter(pred) & Counter(gold)
    same = sum(common.values())
    if same == 0:
        return 0.0
    p = same / len(pred)
    r = same / len(gold)
    return 2 * p * r / (p + r)


def text_scores(pred: str, answers: Sequence[str]) -> dict:
    pn = normalize_answer(pred)
    best = {"qa_f1": 0.0, "exact_match": 0.0, "contains": 0.0}
    for a in answers:
        an = normalize_answer(a)
        best["qa_f1"] = max(best["qa_f1"], token_f1(pn.split(), an.split()))
        best["exact_match"] = max(best["exact_match"], float(pn == an))
        best["contains"] = max(best["contains"], float(bool(an) and an in pn))
    return best


def id_scores(pred: Sequence[int], answers: Sequence[Sequence[int]]) -> dict:
    best = {"qa_f1": 0.0, "exact_match": 0.0, "contains": 0.0}
    pred = list(pred)
    for a in answers:
        a = list(a)
        best["qa_f1"] = max(best["qa_f1"], token_f1(pred, a))
        best["exact_match"] = max(best["exact_match"], float(pred[:len(a)] == a))
        hit = any(pred[i:i + len(a)] == a for i in range(len(pred) - len(a) + 1)) if a else False
        best["contains"] = max(best["contains"], float(hit))
    return best


def _cut_at_stop(ids: list[int], stop_ids: Sequence[Sequence[int]]) -> list[int]:
    end = len(ids)
    for s in stop_ids:
        s = list(s)
        if not s:
            continue
        for i in range(len(ids) - len(s) + 1):
            if ids[i:i + len(s)] == s:
                end = min(end, i)
                break
    return ids[:end]


# ---------------------------------------------------------------- runner

class TaskRunner:
    """Runs local tasks with one cache method (a
    :class:`lm_harness.CacheMethodModel`) and an optional tokenizer."""

    def __init__(self, cache_model, tokenizer=None):
        self.cm = cache_model
        self.tok = tokenizer

    @property
    def device(self):
        return self.cm.model.device

    def _ids(self, doc: dict, key: str, task: LocalTask) -> list[int]:
        if key + "_ids" in doc:
            return [int(i) for i in doc[key + "_ids"]]
        if key not in doc:
            raise ValueError(f"task {task.name!r}: document without {key!r} or {key + '_ids'!r}")
        if self.tok is None:
            raise ValueError(f"task {task.name!r} has text documents: a tokenizer is needed")
        text = doc[key]
        if key == "context" and task.chat_template and getattr(self.tok, "chat_template", None):
            return list(self.tok.apply_chat_template([{"role": "user", "content": text}],
                                                     add_generation_prompt=True, tokenize=True))
        return list(self.tok(text, add_special_tokens=(key == "context"))["input_ids"])

    @torch.no_grad()
    def score_doc(self, task: LocalTask, doc: dict) -> dict:
        ctx = torch.tensor([self._ids(doc, "context", task)], dtype=torch.long,
                           device=self.device)
        if task.kind == "generate":
            out = self.cm.generate(ctx, task.max_new_tokens)[0].tolist()
            if "answers_ids" in doc:
                stops = doc.get("stop_ids") or []
                return id_scores(_cut_at_stop(out, stops), doc["answers_ids"])
            if self.tok is None:
                raise ValueError(f"task {task.name!r} has text answers: a tokenizer is needed")
            text = self.tok.decode(out, skip_special_tokens=True)
            for s in doc.get("stop") or []:
                if s and s in text:
                    text = text[:text.index(s)]
            return text_scores(text, doc["answers"])
        choices = doc.get("choices_ids")
        if choices is None:
            if self.tok is None:
                raise ValueError(f"task {task.name!r} has text choices: a tokenizer is needed")
            choices = [self.tok(c, add_special_tokens=False)["input_ids"] for c in doc["choices"]]
        lls = [self.continuation_logprob(ctx, [int(i) for i in c]) for c in choices]
        gold = int(doc["gold"])
        best = max(range(len(lls)), key=lambda i: lls[i])
        return {"acc": float(best == gold)}

    @torch.no_grad()
    def continuation_logprob(self, ctx: torch.Tensor, cont: list[int]) -> float:
        """Sum of log-probabilities of ``cont`` after ``ctx``: the context is
        prefilled into a new cache of the method, then the continuation runs
        as one decode step over the (reconstructed) cache."""
        if not cont:
            return 0.0
        model = self.cm.model
        cache = self.cm.new_cache()
        first = model(ctx, past_key_values=cache, use_cache=True).logits[0, -1].float()
        lp = torch.log_softmax(first, -1)[cont[0]]
        total = float(lp)
        if len(cont) > 1:
            c = torch.tensor([cont[:-1]], dtype=torch.long, device=ctx.device)
            logits = model(c, past_key_values=cache, use_cache=True).logits[0].float()
            lps = torch.log_softmax(logits, -1)
            tgt = torch.tensor(cont[1:], device=lps.device)
            total += float(lps.gather(1, tgt.view(-1, 1)).sum())
        return total

    def run(self, task: LocalTask, indices: Optional[Sequence[int]] = None) -> dict:
        """Mean metrics over the selected documents (all by default), with
        ``score`` = the task's primary metric."""
        idx = list(range(len(task.docs))) if indices is None else list(indices)
        if not idx:
            raise ValueError(f"task {task.name!r}: no documents selected")
        sums: dict[str, float] = {}
        for i in idx:
            for k, v in self.score_doc(task, task.docs[i]).items():
                sums[k] = sums.get(k, 0.0) + v
        out = {k: v / len(idx) for k, v in sums.items()}
        out["score"] = out[task.metric]
        out["docs"] = len(idx)
        return out
