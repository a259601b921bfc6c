"""DuoAttention head scores computed on the fly from a model and sample texts.

The reference's experimental scorer
(kvserve_v1/compression/config/duo_config/get_config.py:14-86, and the
offline copy kvserve_v1/offline_search/duo_config/duo_config.py:10-86)
rates every (layer, KV head) by how far back its attention reaches.  Per
sample and layer:

1. the mean query and the mean key of each head over the sample's tokens
   (the projections of the layer's normalised input, biases included);
2. both repeated over ``q_len`` positions and rotated by the model's RoPE;
3. the softmax of the last query against all ``q_len`` keys (scaled by
   ``1/sqrt(head_dim)``);
4. the score is the mean of that distribution's cumulative sum (the area under
   the cumulative attention curve): heads that look at the oldest positions
   score near 1, heads that only look at the newest positions near
   ``1/q_len``; query heads are averaged within their KV group, and the
   scores are averaged over samples.

The reference samples BookSum texts; no dataset is reachable offline, so the
caller passes the samples (token-id tensors, or texts with a tokenizer).
Differences of form, not of definition: the layer inputs are taken by forward
pre-hooks on the attention modules during one pass of the decoder body (no
stored hidden states, no LM head), and only the last query position is
rotated, since step 3 uses only it; the means and everything after them run
in fp32.

``python -m kvserve_hpdps_b200.offline.duo_scores --model <path> --texts f.txt
--out <model>_scores.csv`` writes a table that
:func:`kvserve_hpdps_b200.compression.head_scores.get_scores_from_csv` reads.
"""

from __future__ import annotations

import argparse
import importlib
import math
from typing import Iterable, Optional, Sequence, Union

import torch

Sample = Union[torch.Tensor, Sequence[int], str]


def _rope_fn(attn_module):
    """The ``apply_rotary_pos_emb`` of the module's own modeling file."""
    return getattr(importlib.import_module(type(attn_module).__module__), "apply_rotary_pos_emb")


def _to_ids(sample: Sample, tokenizer, max_tokens: int, device) -> torch.Tensor:
    if isinstance(sample, str):
        if tokenizer is None:
            raise ValueError("text samples need a tokenizer")
        ids = tokenizer(sample, return_tensors="pt", max_length=max_tokens,
                        truncation=True)["input_ids"][0]
    else:
        ids = torch.as_tensor(sample, dtype=torch.long).reshape(-1)
    return ids[:max_tokens].to(device).view(1, -1)


@torch.no_grad()
def layer_scores(q_mean: torch.Tensor, k_mean: torch.Tensor, cos: torch.Tensor,
                 sin: torch.Tensor, rope) -> torch.Tensor:
    """Scores of one layer from its mean query ``[q_heads, d]`` and mean key
    ``[kv_heads, d]`` (fp32) and the rotary tables ``[1, q_len, d]``:
    ``[kv_heads]``."""
    n_q, d = q_mean.shape
    n_kv = k_mean.shape[0]
    q_len = cos.shape[1]
    q = q_mean.view(1, n_q, 1, d)
    k = k_mean.view(1, n_kv, 1, d).expand(1, n_kv, q_len, d)
    q_last, _ = rope(q, q, cos[:, -1:], sin[:, -1:])
    _, k_rot = rope(k, k, cos, sin)
    k_rot = k_rot.repeat_interleave(n_q // n_kv, dim=1)  # [1, n_q, q_len, d]
    logits = torch.matmul(k_rot, q_last.transpose(2, 3)).squeeze(-1) / math.sqrt(d)
    w = torch.softmax(logits[0], dim=-1)  # [n_q, q_len]
    area = torch.cumsum(w, dim=-1).mean(dim=-1)
    return area.view(n_kv, n_q // n_kv).mean(dim=1)


@torch.no_grad()
def duo_scores_on_the_fly(model, samples: Iterable[Sample], q_len: int = 1024,
                          max_tokens: int = 2048, tokenizer=None) -> torch.Tensor:
    """``[num_layers, num_kv_heads]`` float32 scores of a Hugging Face
    Llama/Qwen2-style causal LM (``model.model.layers[i].self_attn`` with
    ``q_proj``/``k_proj`` and ``model.model.rotary_emb``)."""
    body = model.model
    layers = body.layers
    cfg = model.config
    n_q = int(cfg.num_attention_heads)
    n_kv = int(cfg.num_key_value_heads)
    dev = next(model.parameters()).device
    means: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
    handles = []
    for idx, layer in enumerate(layers):
        def hook(module, args, kwargs, idx=idx):
            h = args[0] if args else kwargs["hidden_states"]
            d = module.head_dim
            q = module.q_proj(h).float().mean(dim=1)[0].view(n_q, d)
            k = module.k_proj(h).float().mean(dim=1)[0].view(n_kv, d)
            means[idx] = (q, k)
            return None
        handles.append(layer.self_attn.register_forward_pre_hook(hook, with_kwargs=True))
    scores = torch.zeros((len(layers), n_kv), dtype=torch.float32)
    n = 0
    try:
        for sample in samples:
            ids = _to_ids(sample, tokenizer, max_tokens, dev)
            if ids.numel() == 0:
                continue
            means.clear()
            body(input_ids=ids, use_cache=False)
            for idx, layer in enumerate(layers):
                q, k = means[idx]
                pos = torch.arange(q_len, device=q.device).view(1, -1)
                cos, sin = body.rotary_emb(q.view(1, 1, 1, -1), pos)
                s = layer_scores(q, k, cos.float(), sin.float(), _rope_fn(layer.self_attn))
                scores[idx] += s.cpu()
            n += 1
    finally:
        for h in handles:
            h.remove()
    if n == 0:
        raise ValueError("no non-empty samples")
    return scores / n


def save_scores_csv(scores: torch.Tensor, path: str) -> None:
    """One row per layer, one column per KV head, no header or index (the
    layout of the shipped tables)."""
    with open(path, "w") as f:
        for row in torch.as_tensor(scores, dtype=torch.float32).tolist():
            f.write(",".join(repr(float(v)) for v in row) + "\n")


def _read_texts(paths: Sequence[str]) -> list[str]:
    """Texts from files: paragraphs separated by blank lines."""
    out = []
    for p in paths:
        with open(p) as f:
            out += [t.strip() for t in f.read().split("\n\n") if t.strip()]
    return out


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(description="DuoAttention scores on the fly")
    ap.add_argument("--model", required=True,
                    help="local Hugging Face checkpoint, or random:<arch> (random weights)")
    ap.add_argument("--texts", nargs="*", default=[],
                    help="text files (paragraphs separated by blank lines)")
    ap.add_argument("--random-samples", type=int, default=4,
                    help="random token samples when no text file is given")
    ap.add_argument("--num-samples", type=int, default=0, help="0 = all")
    ap.add_argument("--q-len", type=int, default=1024)
    ap.add_argument("--max-tokens", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=None, help="random:<arch> layer count")
    ap.add_argument("--hidden", type=int, default=None, help="random:<arch> hidden size")
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    tok = None
    if args.model.startswith("random:"):
        from kvserve_hpdps_b200.offline.cr_methods import random_model
        model, _ = random_model(args.model[len("random:"):], layers=args.layers,
                                hidden=args.hidden)
    else:
        from transformers import AutoModelForCausalLM, AutoTokenizer
        model = AutoModelForCausalLM.from_pretrained(args.model, dtype=torch.bfloat16).eval()
        if torch.cuda.is_available():
            model = model.cuda()
        tok = AutoTokenizer.from_pretrained(args.model)
    samples: list = _read_texts(args.texts)
    if not samples:
        g = torch.Generator().manual_seed(0)
        samples = [torch.randint(0, int(model.config.vocab_size), (args.max_tokens,),
                                 generator=g) for _ in range(args.random_samples)]
    if args.num_samples > 0:
        samples = samples[:args.num_samples]
    scores = duo_scores_on_the_fly(model, samples, args.q_len, args.max_tokens, tok)
    if args.out:
        save_scores_csv(scores, args.out)
    print(scores.numpy())
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
