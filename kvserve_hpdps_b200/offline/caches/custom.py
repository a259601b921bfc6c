"""KVServe's own offline cache: transform, head-score split into LOW and
HIGH precision heads, min-max quantization per head class, rebuild at the
first decode step (reference cache_utils.py:288-692).

Config fields keep the reference's names and checks: ``transform_type`` in
none | hadamard | affine, ``scores`` ([layers, kv_heads] head scores),
``heads_selection`` (fraction of LOW heads, lowest scores first),
high/low key/value max values in [1, 255] with high >= low, and
``axis_key`` / ``axis_value`` (reduction axes of ``[batch, heads, tokens,
head_dim]``: the default keys reduce over tokens (per-channel scales),
values over heads and head_dim (per-token scales)).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch

from kvserve_hpdps_b200.offline.caches.common import (OfflineCache, OfflineLayer, coded_bytes,
                                                      low_precision_mask, minmax_codes,
                                                      minmax_values, tensor_bytes)
from kvserve_hpdps_b200.offline.caches.transforms import make_transform


@dataclass
class CustomCacheConfig:
    transform_type: str = "none"
    scores: Optional[torch.Tensor] = None
    heads_selection: float = 0.5
    high_key_max_value: int = 64
    high_value_max_value: int = 64
    low_key_max_value: int = 32
    low_value_max_value: int = 32
    axis_key: list = field(default_factory=lambda: [2])
    axis_value: list = field(default_factory=lambda: [1, 3])
    device: str = "cpu"
    comp_cr: bool = False
    base_seed: int = 0x3333
    affine_params_path: Optional[str] = None

    def __post_init__(self):
        self.validate()

    def validate(self) -> None:
        if self.transform_type not in ("none", "hadamard", "affine"):
            raise ValueError("transform_type should be in ['none', 'hadamard', 'affine']")
        if not 0.0 <= float(self.heads_selection) <= 1.0:
            raise ValueError("heads_selection should be between 0 and 1")
        for hi, lo, what in ((self.high_key_max_value, self.low_key_max_value, "key"),
                             (self.high_value_max_value, self.low_value_max_value, "value")):
            if hi < lo:
                raise ValueError(f"high_{what}_max_value should be >= low_{what}_max_value")
        for v in (self.high_key_max_value, self.high_value_max_value, self.low_key_max_value,
                  self.low_value_max_value):
            if not 0 < int(v) < 256:
                raise ValueError("max values should be between 1 and 255")
        for ax in list(self.axis_key) + list(self.axis_value):
            if not 0 <= int(ax) <= 3:
                raise ValueError("axes index [batch, heads, tokens, head_dim] (0..3)")


class _CustomLayer(OfflineLayer):
    def update(self, key_states, value_states, *args, **kwargs):
        self.seen += key_states.shape[-2]
        c: CustomCache = self.owner
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
            self.packed = c._pack(self.layer_idx, key_states, value_states)
            return key_states, value_states
        if getattr(self, "packed", None) is not None:
            self.keys, self.values = c._unpack(self.layer_idx, self.packed)
            self.packed = None
        self.keys = torch.cat([self.keys, key_states], dim=-2)
        self.values = torch.cat([self.values, value_states], dim=-2)
        return self.keys, self.values


class CustomCache(OfflineCache):
    def __init__(self, config: CustomCacheConfig):
        super().__init__(lambda owner, i: _CustomLayer(owner, i))
        self.config = config
        self.transform = make_transform(config.transform_type, config.base_seed,
                                        params_path=config.affine_params_path,
                                        device=config.device)
        self.scores_mask = low_precision_mask(config.scores, config.heads_selection)
        self.packs: dict[int, dict] = {}  # layer -> last packed form (kept for CR)

    def _layer_mask(self, layer_idx: int, num_heads: int, device) -> torch.Tensor:
        if self.scores_mask is None:
            return torch.zeros(num_heads, dtype=torch.bool, device=device)
        return self.scores_mask[layer_idx].to(device)

    def _pack(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> dict:
        cfg = self.config
        kt = self.transform.transform(k, layer_idx, "k")
        vt = self.transform.transform(v, layer_idx, "v")
        low = self._layer_mask(layer_idx, k.shape[1], k.device)
        pack = {"low": low, "shape": tuple(k.shape), "dtype": k.dtype}
        for name, x, lo_max, hi_max, axes in (
                ("k", kt, cfg.low_key_max_value, cfg.high_key_max_value, cfg.axis_key),
                ("v", vt, cfg.low_value_max_value, cfg.high_value_max_value, cfg.axis_value)):
            pack[name + "_low"] = minmax_codes(x[:, low].contiguous(), lo_max, axes)
            pack[name + "_high"] = minmax_codes(x[:, ~low].contiguous(), hi_max, axes)
        self.packs[layer_idx] = pack
        return pack

    def _unpack(self, layer_idx: int, pack: dict):
        low = pack["low"]
        out = []
        for name in ("k", "v"):
            x = torch.empty(pack["shape"], dtype=pack["dtype"], device=low.device)
            x[:, low] = minmax_values(*pack[name + "_low"]).to(x.dtype)
            x[:, ~low] = minmax_values(*pack[name + "_high"]).to(x.dtype)
            out.append(self.transform.inverse(x, layer_idx, name))
        if self.config.comp_cr and not self.compression_ratio:
            self.compression_ratio = self.compute_compression_ratio()
        return out[0], out[1]

    def compute_compression_ratio(self) -> float:
        """Original bf16 bytes of the prefill KV over (coded codes + metadata)."""
        if not self.packs:
            return 0.0
        codes, metas, orig = [], [], 0
        for p in self.packs.values():
            b, h, t, d = p["shape"]
            orig += 2 * b * h * t * d * torch.empty((), dtype=p["dtype"]).element_size()
            for key in ("k_low", "k_high", "v_low", "v_high"):
                codes.append(p[key][0])
                metas.append(p[key][1])
        comp = coded_bytes(codes) + tensor_bytes(metas)
        return round(orig / comp, 4) if comp else 0.0
