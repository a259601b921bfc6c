"""Accuracy harness for KV-cache methods on Hugging Face causal LMs.

The reference scores a cache configuration with lm-eval tasks run through a
custom ``HFLM`` subclass that swaps the model's KV cache
(kvserve_v1/offline_search/evaluation/lm_eval/lm_wrapper.py:21-219), and
normalises the task score against the default cache (acc_evaluator.py:
183-242).  No datasets are reachable offline, so the harness here measures
the same thing on any prompt set: greedy continuations with a method's cache
against the default cache, plus the next-token distribution after the first
reconstructed step.  ``register_lm_eval()`` adds the lm-eval model class when
lm-eval is installed.

Methods: ``default`` (plain ``DynamicCache``), ``custom`` (KVServe's
hybrid-precision cache), ``kivi``, ``cachegen``, ``duoattn``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Optional, Sequence

import torch

METHODS = ("default", "custom", "kivi", "cachegen", "duoattn")


def make_cache(method: str, num_layers: int, scores: Optional[torch.Tensor] = None,
               **params: Any):
    """A fresh cache object for one generation call."""
    from transformers import DynamicCache

    from kvserve_hpdps_b200.offline import caches as C
    if method == "default":
        return DynamicCache()
    if method == "custom":
        return C.CustomCache(C.CustomCacheConfig(scores=scores, **params))
    if method == "kivi":
        return C.KIVICache(C.KIVICacheConfig(**params))
    if method == "cachegen":
        return C.CacheGenCache(C.CacheGenCacheConfig(model_layers=num_layers, **params))
    if method == "duoattn":
        return C.DuoAttentionCache(C.DuoAttentionCacheConfig(scores=scores, **params))
    raise ValueError(f"unknown cache method {method!r}; expected one of {METHODS}")


class CacheMethodModel:
    """A causal LM whose every generation call runs with a new cache of one
    method (DuoAttention also gets the query hooks it needs)."""

    def __init__(self, model, method: str = "default", scores: Optional[torch.Tensor] = None,
                 **params: Any):
        self.model = model
        self.method = method
        self.scores = scores
        self.params = params
        self.num_layers = int(model.config.num_hidden_layers)
        self._hooks = []
        if method == "duoattn":
            from kvserve_hpdps_b200.offline.caches import enable_query_capture
            self._hooks = enable_query_capture(model)
        self.last_cache = None

    def close(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []

    def new_cache(self):
        self.last_cache = make_cache(self.method, self.num_layers, self.scores, **self.params)
        return self.last_cache

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 32,
                 attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        out = self.model.generate(input_ids, attention_mask=attention_mask,
                                  max_new_tokens=max_new_tokens, do_sample=False,
                                  past_key_values=self.new_cache(),
                                  pad_token_id=self.model.config.pad_token_id or 0)
        return out[:, input_ids.shape[1]:]

    @torch.no_grad()
    def second_step_logits(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Logits after prefill + one decode step, the first forward that
        attends to the method's reconstructed KV."""
        cache = self.new_cache()
        out = self.model(input_ids, past_key_values=cache, use_cache=True)
        nxt = out.logits[:, -1:].argmax(-1)
        out2 = self.model(nxt, past_key_values=cache, use_cache=True)
        return out2.logits[:, -1].float()


@dataclass
class MethodScore:
    method: str
    accuracy: float            # greedy-token agreement with the default cache, x100
    top1_agreement: float      # first reconstructed step, fraction of prompts
    kl: float                  # mean KL(default || method) of that step
    compression_ratio: float

    def as_dict(self) -> dict:
        return dict(self.__dict__)


@torch.no_grad()
def evaluate_method(model, prompts: Sequence[torch.Tensor], method: str,
                    scores: Optional[torch.Tensor] = None, max_new_tokens: int = 16,
                    **params: Any) -> MethodScore:
    """Score one cache method on ``prompts`` (1-D token-id tensors)."""
    base = CacheMethodModel(model, "default")
    test = CacheMethodModel(model, method, scores, **params)
    try:
        agree = total = top1 = 0
        kl = 0.0
        crs = []
        for p in prompts:
            ids = p.view(1, -1).to(model.device)
            ref = base.generate(ids, max_new_tokens)
            got = test.generate(ids, max_new_tokens)
            n = min(ref.shape[1], got.shape[1])
            agree += int((ref[:, :n] == got[:, :n]).sum())
            total += n
            cache = test.last_cache
            if hasattr(cache, "compute_compression_ratio"):
                crs.append(float(cache.compute_compression_ratio()))
            lr = base.second_step_logits(ids)
            lt = test.second_step_logits(ids)
            top1 += int((lr.argmax(-1) == lt.argmax(-1)).sum())
            pr = torch.log_softmax(lr, -1)
            pt = torch.log_softmax(lt, -1)
            kl += float((pr.exp() * (pr - pt)).sum(-1).mean())
        n_p = max(1, len(prompts))
        return MethodScore(method, 100.0 * agree / max(1, total), top1 / n_p, kl / n_p,
                           sum(crs) / len(crs) if crs else 1.0)
    finally:
        test.close()


_CONFIGS = {"custom": "CustomCacheConfig", "kivi": "KIVICacheConfig",
            "cachegen": "CacheGenCacheConfig", "duoattn": "DuoAttentionCacheConfig"}


def split_cache_args(cache_type: str, kwargs: dict) -> tuple[dict, Optional[str], dict]:
    """Split lm-eval ``model_args`` into (cache parameters, score-table name,
    the rest for ``HFLM``).  A cache parameter is a field of the method's
    config, written bare as the reference's wrapper takes it
    (``transform_type=hadamard``) or prefixed (``cache_transform_type=...``);
    ``scores`` / ``scores_model`` name a head-score table (model name or
    CSV).  ``model_layers`` is filled in from the model for CacheGen."""
    import dataclasses

    from kvserve_hpdps_b200.offline import caches as C
    if cache_type not in METHODS:
        raise ValueError(f"unknown cache method {cache_type!r}; expected one of {METHODS}")
    fields = set()
    if cache_type in _CONFIGS:
        fields = {f.name for f in dataclasses.fields(getattr(C, _CONFIGS[cache_type]))}
    fields -= {"scores", "model_layers"}
    params, rest, scores = {}, {}, None
    for k, v in kwargs.items():
        bare = k[len("cache_"):] if k.startswith("cache_") else k
        if bare in ("scores", "scores_model"):
            scores = v
        elif bare in fields:
            params[bare] = v
        else:
            rest[k] = v
    return params, scores, rest


def register_lm_eval(name: str = "my_custom_model"):
    """Register an lm-eval model class (``HFLM`` subclass) that generates
    with a cache method, under the reference's model name by default:
    ``--model my_custom_model --model_args pretrained=...,cache_type=custom,
    transform_type=hadamard,heads_selection=0.5,...`` (see
    :func:`split_cache_args`).  Needs the ``lm_eval`` package."""
    try:
        from lm_eval.api.registry import register_model
        from lm_eval.models.huggingface import HFLM
    except ImportError as e:  # not installed in every environment
        raise RuntimeError("lm-eval is not installed; use evaluate_method() instead") from e

    @register_model(name)
    class KVServeCacheLM(HFLM):
        def __init__(self, *args, cache_type: str = "default", **kwargs):
            params, scores_name, rest = split_cache_args(cache_type, kwargs)
            super().__init__(*args, **rest)
            from kvserve_hpdps_b200.compression.head_scores import get_scores_from_csv
            if isinstance(scores_name, torch.Tensor):  # a table passed in-process
                scores = scores_name
            else:
                scores = get_scores_from_csv(scores_name) if scores_name else None
            self._kvs = CacheMethodModel(self.model, cache_type, scores, **params)

        def _model_generate(self, context, max_length, stop, **generation_kwargs):
            generation_kwargs.pop("do_sample", None)
            return self.model.generate(input_ids=context, max_length=max_length,
                                       do_sample=False, past_key_values=self._kvs.new_cache(),
                                       pad_token_id=self.tokenizer.pad_token_id or 0,
                                       **generation_kwargs)

    return KVServeCacheLM
