"""Shared pieces of the offline KV caches: min-max codes over tensor axes,
the per-layer cache base class and the compression-ratio measurement.

The caches plug into Hugging Face ``transformers`` (5.x ``Cache`` API): a
cache object owns one layer object per decoder layer, and every attention
layer calls ``cache.update(key_states, value_states, layer_idx)`` with
``[batch, kv_heads, tokens, head_dim]`` states.  The caches here compress at
prefill (the first update of a layer) and rebuild at the first decode step,
the offline-evaluation protocol of the reference
(kvserve_v1/offline_search/src/cache/cache_utils.py:385-436): the prefill
attention sees exact KV, every later token attends to the reconstruction.
"""

from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch
from transformers.cache_utils import Cache, DynamicLayer


def minmax_codes(x: torch.Tensor, max_value: int, dims: Sequence[int]):
    """Asymmetric min-max codes of ``x`` reduced over ``dims``, computed in
    ``x``'s dtype: ``scale = max(max - min, 1e-5) / (max_value - 1)``,
    ``q = clamp(round((x - min) / scale), 0, max_value)``.  Returns the uint8
    codes and ``stack([min, scale])`` (keepdim shapes)."""
    dims = tuple(int(d) % x.dim() for d in dims)
    if x.numel() == 0:
        shape = [1 if i in dims else s for i, s in enumerate(x.shape)]
        z = torch.zeros(shape, dtype=x.dtype, device=x.device)
        return x.to(torch.uint8), torch.stack([z, z])
    lo = torch.amin(x, dim=dims, keepdim=True)
    hi = torch.amax(x, dim=dims, keepdim=True)
    scale = (hi - lo).clamp(min=1e-5) / (max_value - 1)
    q = ((x - lo) / scale).round().clamp(0, max_value).to(torch.uint8)
    return q, torch.stack([lo.to(x.dtype), scale.to(x.dtype)])


def minmax_values(codes: torch.Tensor, meta: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`minmax_codes`: ``q * scale + min`` in the meta dtype."""
    if codes.numel() == 0:
        return codes.to(meta.dtype)
    return codes.to(meta.dtype) * meta[1] + meta[0]


def low_precision_mask(scores: Optional[torch.Tensor], ratio: float,
                       device=None) -> Optional[torch.Tensor]:
    """Bool [layers, kv_heads]: True for the ``round(numel * ratio)``
    (layer, head) pairs with the lowest head scores."""
    if scores is None:
        return None
    from kvserve_hpdps_b200.compression.head_scores import head_low_mask
    m = head_low_mask(torch.as_tensor(scores, dtype=torch.float32).cpu(), ratio)
    return m.to(device) if device is not None else m


def coded_bytes(tensors: Sequence[torch.Tensor]) -> int:
    """Bytes of the concatenated uint8 code tensors after this package's
    interleaved rANS coder (the offline stand-in for the reference's nvCOMP
    ANS pass)."""
    from kvserve_hpdps_b200.compression.codec import encode_bytes
    parts = [t.contiguous().view(torch.uint8).reshape(-1) for t in tensors if t.numel()]
    if not parts:
        return 0
    dev = parts[0].device
    flat = torch.cat([p.to(dev) for p in parts])
    return int(encode_bytes(flat, "rans").numel()) - 16  # without the container header


def tensor_bytes(tensors: Sequence[torch.Tensor]) -> int:
    return int(sum(t.numel() * t.element_size() for t in tensors))


class OfflineLayer(DynamicLayer):
    """A decoder layer's cache: tracks the token count itself because the
    compressed layers hold no plain keys between prefill and decode."""

    def __init__(self, owner: "OfflineCache", layer_idx: int):
        super().__init__()
        self.owner = owner
        self.layer_idx = layer_idx
        self.seen = 0

    def get_seq_length(self) -> int:
        return self.seen


class OfflineCache(Cache):
    """Cache whose layers know their index (transformers creates replicated
    layers without arguments, so ``update`` builds them here)."""

    def __init__(self, layer_factory: Callable[["OfflineCache", int], OfflineLayer]):
        super().__init__(layers=[])
        self._layer_factory = layer_factory
        self.compression_ratio = 0.0

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               *args, **kwargs):
        while len(self.layers) <= layer_idx:
            self.layers.append(self._layer_factory(self, len(self.layers)))
        return self.layers[layer_idx].update(key_states, value_states, *args, **kwargs)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        if layer_idx >= len(self.layers):
            return 0
        return self.layers[layer_idx].get_seq_length()
