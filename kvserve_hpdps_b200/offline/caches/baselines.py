"""Offline baseline caches the reference compares against.

* ``KIVICache`` (KIVI, Liu et al. 2024): asymmetric ``nbits`` min-max codes
  in groups of ``q_group_size`` along tokens (axis 2) or channels (axis 3);
  a residual window of the newest tokens stays in full precision and is
  folded into the quantized part whenever it fills (reference
  kivi_utils.py:47-397; its prefill keeps ``len - len % residual`` tokens
  quantized).
* ``CacheGenCache`` (CacheGen, Liu et al. 2024): symmetric absmax codes per
  (batch, token) over heads and head_dim, with per-layer bin counts from
  ``quantization_level`` (keys: the first ~32% / ~63% of layers get more
  bins; values: the first ~15% of layers, at least two) (reference
  cachegen_utils.py:42-300).
* ``DuoAttentionCache`` (DuoAttention, Xiao et al. 2024): the lowest-scored
  (layer, head) pairs are streaming heads that keep only ``sink_size``
  initial and ``recent_size`` latest tokens; the rest of their keys is
  replaced by a fake key on which every current query scores ~-inf (found by
  ``search_hyperplane``), so those tokens get zero attention weight
  (reference duoattn_utils.py:1-206).  It needs the decode queries: call
  :func:`enable_query_capture` on the model first.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from kvserve_hpdps_b200.offline.caches.common import (OfflineCache, OfflineLayer, coded_bytes,
                                                      low_precision_mask, minmax_codes,
                                                      minmax_values, tensor_bytes)


# ---------------------------------------------------------------- KIVI
@dataclass
class KIVICacheConfig:
    nbits: int = 4
    axis_key: int = 2
    axis_value: int = 3
    q_group_size: int = 32
    residual_length: int = 128
    comp_cr: bool = False

    def __post_init__(self):
        if self.nbits not in (1, 2, 3, 4, 8):
            raise ValueError("nbits must be one of 1, 2, 3, 4, 8")
        if self.axis_key not in (2, 3) or self.axis_value not in (2, 3):
            raise ValueError("KIVI groups along tokens (2) or channels (3)")


def _grouped(x: torch.Tensor, axis: int, g: int) -> torch.Tensor:
    b, h, t, d = x.shape
    if axis == 2:
        return x.reshape(b, h, t // g, g, d)
    return x.reshape(b, h, t, d // g, g)


def _kivi_quant(x: torch.Tensor, axis: int, cfg: KIVICacheConfig):
    if x.numel() == 0:
        return x, None, axis
    xg = _grouped(x, axis, cfg.q_group_size)
    red = -2 if axis == 2 else -1
    q, meta = minmax_codes(xg, 2 ** cfg.nbits, [red])
    return q, meta, axis


def _kivi_values(q, meta, axis) -> torch.Tensor:
    if meta is None:
        return q
    x = minmax_values(q, meta)
    b, h = x.shape[:2]
    if axis == 2:
        return x.reshape(b, h, x.shape[2] * x.shape[3], x.shape[4])
    return x.reshape(b, h, x.shape[2], x.shape[3] * x.shape[4])


class _KIVILayer(OfflineLayer):
    def update(self, key_states, value_states, *args, **kwargs):
        cfg: KIVICacheConfig = self.owner.config
        self.seen += key_states.shape[-2]
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
            t = key_states.shape[-2]
            n = (t // cfg.residual_length) * cfg.residual_length
            self.qk = _kivi_quant(key_states[:, :, :n].contiguous(), cfg.axis_key, cfg)
            self.qv = _kivi_quant(value_states[:, :, :n].contiguous(), cfg.axis_value, cfg)
            self.keys = key_states[:, :, n:].contiguous()
            self.values = value_states[:, :, n:].contiguous()
            self.owner._note_prefill(self)
            return key_states, value_states
        if self.owner.config.comp_cr and not self.owner.compression_ratio:
            self.owner.compression_ratio = self.owner.compute_compression_ratio()
        dk = _kivi_values(*self.qk)
        dv = _kivi_values(*self.qv)
        keys = torch.cat([dk.to(key_states.dtype), self.keys, key_states], dim=-2)
        values = torch.cat([dv.to(value_states.dtype), self.values, value_states], dim=-2)
        if self.keys.shape[-2] + 1 >= cfg.residual_length:  # window full: fold it in
            self.qk = _kivi_quant(keys.contiguous(), cfg.axis_key, cfg)
            self.qv = _kivi_quant(values.contiguous(), cfg.axis_value, cfg)
            self.keys = keys[:, :, :0]
            self.values = values[:, :, :0]
        else:
            self.keys = torch.cat([self.keys, key_states], dim=-2)
            self.values = torch.cat([self.values, value_states], dim=-2)
        return keys, values


class KIVICache(OfflineCache):
    def __init__(self, config: KIVICacheConfig):
        super().__init__(lambda owner, i: _KIVILayer(owner, i))
        self.config = config
        self._prefill: list = []

    def _note_prefill(self, layer: _KIVILayer) -> None:
        self._prefill.append((layer.qk, layer.qv, layer.keys, layer.values))

    def compute_compression_ratio(self) -> float:
        """Prefill bf16 bytes over (bit-packed codes + metadata + residual)."""
        from kvserve_hpdps_b200.compression.codec import _bitpack_rows
        orig = packed = 0
        for qk, qv, rk, rv in self._prefill:
            for (q, meta, _), r in ((qk, rk), (qv, rv)):
                elt = r.element_size()
                orig += (q.numel() + r.numel()) * elt
                packed += r.numel() * elt
                if meta is not None:
                    # codes span [0, 2^nbits], so the widest code may need one more bit
                    flat = q.reshape(-1)
                    bits = max(1, int(flat.max()).bit_length())
                    if bits >= 8:
                        packed += flat.numel()
                    else:
                        rows = (flat.numel() + 127) // 128
                        pad = torch.zeros(rows * 128, dtype=torch.uint8, device=flat.device)
                        pad[:flat.numel()] = flat
                        packed += _bitpack_rows(pad.view(rows, 128), bits).numel()
                    packed += tensor_bytes([meta])
        return round(orig / packed, 4) if packed else 0.0


# ---------------------------------------------------------------- CacheGen
@dataclass
class CacheGenCacheConfig:
    model_layers: Optional[int] = None
    quantization_level: int = 1
    high_max_value: int = 32
    mid_max_value: int = 16
    low_max_value: int = 12
    comp_cr: bool = False

    def __post_init__(self):
        if self.model_layers is None:
            raise ValueError("model_layers should be provided")
        if self.quantization_level not in (1, 2, 3):
            raise ValueError("quantization_level should be in [1, 2, 3]")
        if not (0 < self.low_max_value <= self.mid_max_value <= self.high_max_value < 256):
            raise ValueError("need 0 < low <= mid <= high < 256")


def cachegen_bins(cfg: CacheGenCacheConfig) -> list[dict]:
    """Per-layer bin counts {"k": .., "v": ..} for the config's level."""
    n = cfg.model_layers
    k1, k2 = int(n * 0.32), int(n * 0.63)
    v1 = max(2, int(n * 0.15))
    out = []
    for i in range(n):
        if cfg.quantization_level == 1:
            k = cfg.mid_max_value if i < k2 else cfg.low_max_value
            v = cfg.mid_max_value if i < v1 else cfg.low_max_value
        elif cfg.quantization_level == 2:
            k = cfg.high_max_value if i < k1 else cfg.mid_max_value
            v = cfg.high_max_value if i < v1 else cfg.mid_max_value
        else:
            k = v = cfg.high_max_value
        out.append({"k": k, "v": v})
    return out


def _absmax_codes(x: torch.Tensor, bins: int):
    """Codes in [0, 2 * (bins // 2 - 1)] (uint8, so every bin count below
    256 fits) and the per-(batch, token) absmax over heads and head_dim."""
    half = bins // 2 - 1
    amax = torch.amax(x.abs(), dim=(1, 3), keepdim=True)
    q = torch.round(x * (half / amax.clamp_min(1e-12)) + half).clamp(0, 2 * half)
    return q.to(torch.uint8), amax


def _absmax_values(q: torch.Tensor, amax: torch.Tensor, bins: int) -> torch.Tensor:
    half = bins // 2 - 1
    return ((q.float() - half) / half * amax.float()).to(amax.dtype)


class _CacheGenLayer(OfflineLayer):
    def update(self, key_states, value_states, *args, **kwargs):
        owner: CacheGenCache = self.owner
        bins = owner.bins[self.layer_idx]
        self.seen += key_states.shape[-2]
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
            self.qk = _absmax_codes(key_states, bins["k"])
            self.qv = _absmax_codes(value_states, bins["v"])
            return key_states, value_states
        if owner.config.comp_cr and not owner.compression_ratio:
            owner.compression_ratio = owner.compute_compression_ratio()
        self.keys = torch.cat([self.keys, key_states], dim=-2)
        self.values = torch.cat([self.values, value_states], dim=-2)
        dk = _absmax_values(*self.qk, bins["k"])
        dv = _absmax_values(*self.qv, bins["v"])
        return torch.cat([dk, self.keys], dim=-2), torch.cat([dv, self.values], dim=-2)


class CacheGenCache(OfflineCache):
    def __init__(self, config: CacheGenCacheConfig):
        super().__init__(lambda owner, i: _CacheGenLayer(owner, i))
        self.config = config
        self.bins = cachegen_bins(config)

    def compute_compression_ratio(self) -> float:
        """Prefill bf16 bytes over (entropy-coded codes + absmax metadata)."""
        codes, metas, orig = [], [], 0
        for layer in self.layers:
            if not hasattr(layer, "qk"):
                continue
            for q, amax in (layer.qk, layer.qv):
                orig += q.numel() * amax.element_size()
                codes.append(q)
                metas.append(amax)
        comp = coded_bytes(codes) + tensor_bytes(metas)
        return round(orig / comp, 4) if comp else 0.0


# ---------------------------------------------------------------- DuoAttention
def search_hyperplane(x: torch.Tensor, max_iter: int = 1000) -> torch.Tensor:
    """For ``x`` [batch, n, d] find y [batch, d] with <x_i, y> <= 0 for every
    i (perceptron-style updates from the mean), returned scaled as
    ``-1e5 * y / |y|^2`` so that exp(<x_i, y>) underflows to 0."""
    y = x.mean(1)
    for _ in range(max_iter):
        bad = torch.bmm(x, y.unsqueeze(-1)) <= 0
        if not bad.any():
            break
        y = y + (x * bad).sum(1) / bad.sum(1).clamp(min=1)
    return -1e5 * y / y.norm(dim=-1, keepdim=True) ** 2


@dataclass
class DuoAttentionCacheConfig:
    scores: Optional[torch.Tensor] = None
    heads_selection: float = 0.5
    sink_size: int = 128
    recent_size: int = 256
    comp_cr: bool = False

    def __post_init__(self):
        if self.scores is None:
            raise ValueError("scores should be provided")
        if not 0.0 <= float(self.heads_selection) <= 1.0:
            raise ValueError("heads_selection should be between 0 and 1")
        if self.sink_size < 0 or self.recent_size < 0:
            raise ValueError("sink_size and recent_size must be non-negative")


class _DuoLayer(OfflineLayer):
    def update(self, key_states, value_states, *args, **kwargs):
        owner: DuoAttentionCache = self.owner
        self.seen += key_states.shape[-2]
        first = not self.is_initialized
        if first:
            self.lazy_initialization(key_states, value_states)
        self.keys = torch.cat([self.keys, key_states], dim=-2)
        self.values = torch.cat([self.values, value_states], dim=-2)
        if first:
            return self.keys, self.values  # prefill: exact attention
        if owner.config.comp_cr and not owner.compression_ratio:
            owner.compression_ratio = owner.compute_compression_ratio()
        idx = owner.streaming_positions(self.layer_idx, self.keys)
        q = owner.take_query(self.layer_idx)
        if idx is not None and q is not None:
            b, hq, s, d = q.shape
            hk = self.keys.shape[1]
            flat = q.reshape(b, hk, (hq // hk) * s, d).reshape(b * hk, -1, d).float()
            fake = search_hyperplane(flat).view(b, hk, d).to(self.keys.dtype)
            bi, hi, ti = idx
            self.keys[bi, hi, ti] = fake[bi, hi]
        return self.keys, self.values


class DuoAttentionCache(OfflineCache):
    def __init__(self, config: DuoAttentionCacheConfig):
        super().__init__(lambda owner, i: _DuoLayer(owner, i))
        self.config = config
        self.scores_mask = low_precision_mask(config.scores, config.heads_selection)
        self._queries: dict[int, torch.Tensor] = {}

    def offer_query(self, layer_idx: int, query: torch.Tensor) -> None:
        self._queries[int(layer_idx)] = query

    def take_query(self, layer_idx: int) -> Optional[torch.Tensor]:
        return self._queries.pop(int(layer_idx), None)

    def streaming_positions(self, layer_idx: int, keys: torch.Tensor):
        """(batch, head, token) indices of the dropped middle tokens of the
        streaming heads, or None when nothing is dropped."""
        cfg = self.config
        t = keys.shape[-2]
        if t <= cfg.sink_size + cfg.recent_size:
            return None
        heads = self.scores_mask[layer_idx].to(keys.device)
        if not heads.any():
            return None
        drop = torch.zeros(keys.shape[:-1], dtype=torch.bool, device=keys.device)
        drop[:, heads, cfg.sink_size:t - cfg.recent_size] = True
        return torch.nonzero(drop, as_tuple=True)

    def compute_compression_ratio(self) -> float:
        """KV bytes over the bytes the streaming heads keep."""
        orig = kept = 0
        for layer in self.layers:
            if not layer.is_initialized:
                continue
            n = layer.keys.numel() * layer.keys.element_size()
            orig += 2 * n
            idx = self.streaming_positions(layer.layer_idx, layer.keys)
            dropped = 0 if idx is None else idx[0].numel() * layer.keys.shape[-1] * \
                layer.keys.element_size()
            kept += 2 * (n - dropped)
        return round(orig / kept, 4) if kept else 0.0


def enable_query_capture(model) -> list:
    """Give a DuoAttention cache the decode queries of every attention layer.

    A forward pre-hook on each ``self_attn`` module recomputes the rotated
    query from the layer's input (``q_proj`` + the model's rotary
    embedding) and hands it to the cache; the attention code itself is not
    replaced.  Returns the hook handles."""
    import importlib
    handles = []
    for layer in model.model.layers:
        attn = layer.self_attn
        mod = importlib.import_module(type(attn).__module__)
        rope = getattr(mod, "apply_rotary_pos_emb")

        def hook(module, args, kwargs, rope=rope):
            cache = kwargs.get("past_key_values")
            if not isinstance(cache, DuoAttentionCache):
                return None
            hidden = args[0] if args else kwargs["hidden_states"]
            cos, sin = kwargs["position_embeddings"] if "position_embeddings" in kwargs else args[1]
            shape = (*hidden.shape[:-1], -1, module.head_dim)
            q = module.q_proj(hidden).view(shape).transpose(1, 2)
            q, _ = rope(q, q, cos, sin)
            cache.offer_query(module.layer_idx, q)
            return None
        handles.append(attn.register_forward_pre_hook(hook, with_kwargs=True))
    return handles
