"""Compression ratio and accuracy per KV-cache method on one model.

The reference measures CR per method (custom / KIVI / CacheGen /
DuoAttention) with a script per method
(kvserve_v1/offline_search/evaluation/compression_ratio/*_cr.py) and
accuracy with lm-eval.  This tool runs every method's cache on the same
prompts through :mod:`kvserve_hpdps_b200.offline.lm_harness` and prints one
CSV row per method: CR (bytes after this package's codec), greedy-token
agreement with the default cache, top-1 agreement and KL of the first
reconstructed step.

Without checkpoints (no network here), ``--arch`` builds a random-init model
of a named architecture, optionally shrunk (``--layers``, ``--hidden``);
``--model`` loads a local Hugging Face checkpoint directory instead.

Usage::

  python -m kvserve_hpdps_b200.offline.cr_methods --arch Qwen2.5-7B-Instruct \\
      --layers 4 --hidden 512 --tokens 512 --prompts 2
"""

from __future__ import annotations

import argparse
import csv
import sys
from typing import Optional

import torch

DEFAULT_PARAMS = {
    "custom": {"transform_type": "hadamard", "heads_selection": 0.8, "high_key_max_value": 12,
               "high_value_max_value": 8, "low_key_max_value": 6, "low_value_max_value": 4},
    "kivi": {"nbits": 2, "q_group_size": 32, "residual_length": 128},
    "cachegen": {"quantization_level": 1},
    "duoattn": {"heads_selection": 0.5, "sink_size": 64, "recent_size": 256},
}


def random_model(arch: str, layers: Optional[int] = None, hidden: Optional[int] = None,
                 seed: int = 0, dtype=torch.float32, device="cpu"):
    """Random-init causal LM of a named architecture (optionally shrunk:
    fewer layers, smaller hidden size with the same KV-head count and
    head size)."""
    from transformers import AutoConfig, AutoModelForCausalLM  # noqa: F401
    from transformers import LlamaConfig, Qwen2Config

    from kvserve_hpdps_b200.models.specs import get_spec
    s = get_spec(arch)
    L = layers or s.num_layers
    hid = hidden or s.hidden_size
    heads = max(s.num_kv_heads, hid // s.head_dim)
    heads -= heads % s.num_kv_heads
    cls = Qwen2Config if s.hf_architecture.startswith("Qwen2") else LlamaConfig
    cfg = cls(vocab_size=min(s.vocab_size, 32000), hidden_size=heads * s.head_dim,
              intermediate_size=2 * heads * s.head_dim, num_hidden_layers=L,
              num_attention_heads=heads, num_key_value_heads=s.num_kv_heads,
              head_dim=s.head_dim, max_position_embeddings=s.max_position_embeddings,
              rope_theta=s.rope_theta)
    torch.manual_seed(seed)
    from transformers import LlamaForCausalLM, Qwen2ForCausalLM
    model = (Qwen2ForCausalLM if cls is Qwen2Config else LlamaForCausalLM)(cfg)
    return model.to(device=device, dtype=dtype).eval(), s


def run(model, prompts, scores, methods=("custom", "kivi", "cachegen", "duoattn"),
        max_new_tokens: int = 8, params: Optional[dict] = None) -> list[dict]:
    from kvserve_hpdps_b200.offline.lm_harness import evaluate_method
    rows = []
    for m in methods:
        p = dict(DEFAULT_PARAMS.get(m, {}))
        p.update((params or {}).get(m, {}))
        if m == "custom":
            p["device"] = str(model.device)
        r = evaluate_method(model, prompts, m, scores=scores, max_new_tokens=max_new_tokens, **p)
        rows.append(r.as_dict())
    return rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="CR and accuracy per KV-cache method")
    ap.add_argument("--arch", default="Qwen2.5-7B-Instruct")
    ap.add_argument("--model", default=None, help="local HF checkpoint directory")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--hidden", type=int, default=None)
    ap.add_argument("--tokens", type=int, default=512)
    ap.add_argument("--prompts", type=int, default=2)
    ap.add_argument("--new-tokens", type=int, default=8)
    ap.add_argument("--methods", default="custom,kivi,cachegen,duoattn")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    args = ap.parse_args(argv)
    from kvserve_hpdps_b200.compression.head_scores import get_scores_from_csv, synthetic_scores
    dtype = torch.bfloat16 if args.device.startswith("cuda") else torch.float32
    if args.model:
        from transformers import AutoModelForCausalLM
        model = AutoModelForCausalLM.from_pretrained(args.model, torch_dtype=dtype).to(args.device)
        name = args.model
    else:
        model, spec = random_model(args.arch, args.layers, args.hidden, dtype=dtype,
                                   device=args.device)
        name = spec.name
    L = model.config.num_hidden_layers
    H = model.config.num_key_value_heads
    scores = get_scores_from_csv(name)
    if scores is None or tuple(scores.shape) != (L, H):
        scores = synthetic_scores(L, H)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, model.config.vocab_size, (args.tokens,), generator=g)
               for _ in range(args.prompts)]
    rows = run(model, prompts, scores, tuple(args.methods.split(",")), args.new_tokens)
    w = csv.DictWriter(sys.stdout, fieldnames=list(rows[0]))
    w.writeheader()
    w.writerows(rows)
    return 0


if __name__ == "__main__":
    sys.exit(main())
