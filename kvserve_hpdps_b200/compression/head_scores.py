"""Per-(layer, kv-head) importance scores and the hybrid precision masks.

The scores are DuoAttention-style retrieval scores shipped as CSV tables
(``<model>_scores.csv``, one row per layer, one column per KV head).  The
tables in ``data/`` are the reference's data files
(kvserve_v1/compression/config/duo_config/*.csv); they are kept identical so
that the same ``hybrid_ratio`` selects the same low-precision heads on both
sides of a transfer.

Mask rules (reference kvserve_quantizer.py:58-68, kv_hadamard_quant.py:95-108):

* head split: the ``round(L*H*hybrid_ratio)`` (layer, head) pairs with the
  lowest scores are LOW precision, the rest HIGH;
* layer split: the last ``round(L*0.33)`` layers are LOW.  ``round`` is
  Python's round-half-even, and a count of 0 marks every layer LOW, as in the
  reference (``mask[-0:] = True``).

Unlike the reference's fused op, the head mask is sliced to the local heads of
``tp_rank`` (``[tp_rank*H_local, (tp_rank+1)*H_local)``) on every path.
"""

from __future__ import annotations

import os
from functools import lru_cache
from typing import Optional

import torch

_DATA_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "data")

# Architecture aliases: checkpoints of the same architecture share a table.
_ALIASES = {
    "Qwen2.5-7B": "Qwen2.5-7B-Instruct",
    "Qwen2.5-32B": "Qwen2.5-32B-Instruct",
    "Llama-3.1-8B": "Llama-3.1-8B-Instruct",
    "Meta-Llama-3.1-8B-Instruct": "Llama-3.1-8B-Instruct",
    "Llama-3-8B": "Llama-3.1-8B-Instruct",
    "Meta-Llama-3-8B": "Llama-3.1-8B-Instruct",
    "Meta-Llama-3-8B-Instruct": "Llama-3.1-8B-Instruct",
    "Llama-3-8B-Instruct": "Llama-3.1-8B-Instruct",
}


def _read_csv(path: str) -> torch.Tensor:
    rows = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            vals = [v for v in line.split(",") if v.strip() != ""]
            try:
                rows.append([float(v) for v in vals])
            except ValueError:
                continue
    if not rows:
        raise ValueError(f"empty score table {path}")
    width = min(len(r) for r in rows)
    return torch.tensor([r[:width] for r in rows], dtype=torch.float32)


@lru_cache(maxsize=32)
def _load_cached(model_name: str) -> Optional[torch.Tensor]:
    base = model_name.strip("/").split("/")[-1]
    names = [base]
    if base in _ALIASES:
        names.append(_ALIASES[base])
    for name in names:
        fname = f"{name}_scores.csv"
        for path in (os.path.join(_DATA_DIR, fname), os.path.join(os.getcwd(), fname), fname):
            if os.path.exists(path):
                return _read_csv(path)
    return None


def get_scores_from_csv(model_name: Optional[str]) -> Optional[torch.Tensor]:
    """[num_layers, num_kv_heads] float32 scores, or None if no table exists.

    Search order (reference get_config.py:90-117): package data dir, current
    directory, bare relative path; then the architecture alias table.
    """
    if not model_name:
        return None
    t = _load_cached(str(model_name))
    return None if t is None else t.clone()


def synthetic_scores(num_layers: int, num_heads: int, seed: int = 0x5EED) -> torch.Tensor:
    """Deterministic stand-in table for architectures without a shipped CSV."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed ^ (num_layers << 8) ^ num_heads)
    return torch.rand((num_layers, num_heads), generator=g, dtype=torch.float32)


class DuoConfigGenerator:
    """The reference's entry points for the scores
    (kvserve_v1/compression/config/duo_config/get_config.py:8-117):
    ``get_scores_from_csv`` reads a shipped or saved table,
    ``duo_attention_on_the_fly`` computes one from a model and samples
    (:func:`kvserve_hpdps_b200.offline.duo_scores.duo_scores_on_the_fly`)."""

    @staticmethod
    def duo_attention_on_the_fly(model, samples, q_len: int = 1024, max_tokens: int = 2048,
                                 tokenizer=None) -> torch.Tensor:
        from kvserve_hpdps_b200.offline.duo_scores import duo_scores_on_the_fly
        return duo_scores_on_the_fly(model, samples, q_len, max_tokens, tokenizer)

    @classmethod
    def get_scores_from_csv(cls, model_name: str) -> Optional[torch.Tensor]:
        return get_scores_from_csv(model_name)


def head_low_mask(scores: torch.Tensor, hybrid_ratio: float) -> torch.Tensor:
    """Bool [L, H]: True where the (layer, head) pair is LOW precision."""
    n_low = round(scores.numel() * float(hybrid_ratio))
    mask = torch.zeros(scores.numel(), dtype=torch.bool)
    if n_low > 0:
        order = torch.argsort(scores.flatten(), stable=True)[:n_low]
        mask[order] = True
    return mask.view_as(scores)


def layer_low_mask(num_layers: int) -> torch.Tensor:
    """Bool [L]: the last round(L*0.33) layers are LOW (all when that is 0)."""
    mask = torch.zeros(num_layers, dtype=torch.bool)
    n = round(num_layers * 0.33)
    mask[-n:] = True
    return mask


def slice_for_tp(mask: torch.Tensor, num_local_heads: int, tp_rank: int = 0,
                 tp_size: Optional[int] = None) -> torch.Tensor:
    """Columns of a [L, H_total] mask owned by ``tp_rank``.

    Raises when the table width is not ``tp_size * num_local_heads``
    (reference kvserve_quantizer.py:76-103).
    """
    total = mask.shape[1]
    if total == num_local_heads:
        return mask
    if total % num_local_heads != 0:
        raise ValueError(f"head table has {total} heads, tensor has {num_local_heads}")
    inferred = total // num_local_heads
    tp = tp_size or inferred
    if tp * num_local_heads != total:
        raise ValueError(f"TP mismatch: tp_size={tp} local_heads={num_local_heads} total={total}")
    if not 0 <= tp_rank < tp:
        raise ValueError(f"invalid tp_rank={tp_rank} for tp_size={tp}")
    return mask[:, tp_rank * num_local_heads:(tp_rank + 1) * num_local_heads]


class HybridPrecisionPlan:
    """Per-layer, per-local-head quantization level counts for K and V.

    ``key_levels[l, h]`` / ``value_levels[l, h]`` hold the quantizer's
    ``max_value`` (a LEVEL count: codes span 0..max_value-1, scale =
    range/(max_value-1)) for layer l and local head h.  Without a score table
    every head uses the HIGH values, as the reference's fused op does
    (kv_hadamard_quant.py:109-112, :1338-1342).
    """

    def __init__(self, num_layers: Optional[int], num_local_heads: int,
                 model_name: Optional[str], hybrid_ratio: float,
                 high_key: float, high_value: float, low_key: float, low_value: float,
                 split_type: str = "head", tp_rank: int = 0, tp_size: int = 1):
        self.num_local_heads = int(num_local_heads)
        self.high_key, self.high_value = float(high_key), float(high_value)
        self.low_key, self.low_value = float(low_key), float(low_value)
        self.split_type = split_type
        scores = get_scores_from_csv(model_name)
        self.has_table = scores is not None
        if scores is None:
            L = int(num_layers or 1)
            self.low = torch.zeros((L, self.num_local_heads), dtype=torch.bool)
        else:
            if split_type == "head":
                full = head_low_mask(scores, hybrid_ratio)
                self.low = slice_for_tp(full, self.num_local_heads, tp_rank, tp_size)
            else:
                lm = layer_low_mask(scores.shape[0])
                self.low = lm[:, None].expand(scores.shape[0], self.num_local_heads).clone()
        self.num_layers = self.low.shape[0]
        lowf = self.low.to(torch.float32)
        self.key_levels = lowf * self.low_key + (1 - lowf) * self.high_key
        self.value_levels = lowf * self.low_value + (1 - lowf) * self.high_value

    def layer_index(self, layer_id: int) -> int:
        # Layers past the table reuse the last row (a stacked run longer than
        # the table, e.g. a random-init model with more layers).
        return min(int(layer_id), self.num_layers - 1)

    def key_levels_for(self, layer_id: int) -> torch.Tensor:
        return self.key_levels[self.layer_index(layer_id)]

    def value_levels_for(self, layer_id: int) -> torch.Tensor:
        return self.value_levels[self.layer_index(layer_id)]

    def value_groups_for(self, layer_id: int) -> tuple[list[int], list[list[int]]]:
        """Heads with equal value level share one per-token scale.  Group ids
        follow first appearance (reference kv_hadamard_quant.py:1180-1191).
        Returns (group_of_head, heads_of_group)."""
        lv = self.value_levels_for(layer_id).tolist()
        gid: dict[float, int] = {}
        group_of_head, heads = [], []
        for h, v in enumerate(lv):
            if v not in gid:
                gid[v] = len(gid)
                heads.append([])
            group_of_head.append(gid[v])
            heads[gid[v]].append(h)
        return group_of_head, heads
