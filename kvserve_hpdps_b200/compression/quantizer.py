"""Quantizer stage of the generic pipeline (hybrid head/layer precision).

Semantics of the reference quantizer (kvserve_v1/compression/quantizer/*),
kept exactly because the generic pipeline exists for configurations that
must reproduce it:

* asymmetric min-max quantization in the tensor's dtype:
  ``scale = (max - min).clamp(1e-5) / (max_value - 1)``,
  ``q = clamp(round((x - min) / scale), 0, max_value)`` (round half to
  even), dequantization ``q * scale + min``;
* axis ``channel`` reduces over (blocks, block_size), ``token`` over
  (heads, head_dim), ``tensor`` over everything;
* ``split_type="head"``: the lowest-scored (layer, head) pairs (by
  ``hybrid_ratio``) use the LOW max values, the others HIGH; the quantized
  tensor holds the LOW heads first, then the HIGH heads; ``"layer"``: the
  last third of the layers is LOW.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

from kvserve_hpdps_b200.compression.components import Quantizer
from kvserve_hpdps_b200.compression.config import QUANTIZER_DEFAULTS, validate_quantizer_config
from kvserve_hpdps_b200.compression.head_scores import (get_scores_from_csv, head_low_mask,
                                                        layer_low_mask, slice_for_tp,
                                                        synthetic_scores)

_AXES = {"channel": (0, 1), "token": (2, 3), "tensor": (0, 1, 2, 3)}


def _levels(max_value: float, x: torch.Tensor, axis: str) -> tuple[torch.Tensor, dict]:
    """Quantized levels in ``x``'s dtype (whole numbers in [0, max_value])
    and the metadata."""
    dtype = str(x.dtype).replace("torch.", "")
    dims = _AXES[axis]
    mx = torch.amax(x, dim=dims, keepdim=True)
    mn = torch.amin(x, dim=dims, keepdim=True)
    scale = (mx - mn).clamp_(min=1e-5).div_(max_value - 1)
    q = x.sub(mn).div_(scale).round_().clamp_(0, max_value)
    return q, {"min_val": mn.to(x.dtype), "quant_scale": scale.to(x.dtype),
               "original_dtype": dtype, "quant_dtype": "uint8"}


def quantize(max_value: float, x: torch.Tensor, axis: str) -> tuple[torch.Tensor, dict]:
    if x.numel() == 0:
        return x.to(torch.uint8), {"min_val": None, "quant_scale": None,
                                   "original_dtype": str(x.dtype).replace("torch.", ""),
                                   "quant_dtype": "uint8"}
    q, meta = _levels(max_value, x, axis)
    return q.to(torch.uint8), meta


def dequantize(q: torch.Tensor, meta: dict) -> torch.Tensor:
    dtype = getattr(torch, meta.get("original_dtype", "bfloat16"))
    if meta["min_val"] is None:
        return q.to(dtype)
    return q.to(dtype) * meta["quant_scale"] + meta["min_val"]


class KVServeQuantizer(Quantizer):
    def __init__(self, **kwargs: Any):
        cfg = dict(QUANTIZER_DEFAULTS)
        cfg.update({k: v for k, v in kwargs.items() if v is not None})
        for k in ("model_name", "hybrid_ratio", "high_key_max_value", "high_value_max_value",
                  "low_key_max_value", "low_value_max_value", "axis_key", "axis_value",
                  "split_type"):
            setattr(self, k, cfg[k])
        self.tensor_parallel_size = int(kwargs.get("tensor_parallel_size", 1) or 1)
        self.tp_rank = int(kwargs.get("tp_rank", 0) or 0)
        self.num_layers = kwargs.get("num_layers")
        self.validate()
        self._build_masks()

    def validate(self) -> None:
        validate_quantizer_config({k: getattr(self, k) for k in (
            "hybrid_ratio", "high_key_max_value", "high_value_max_value", "low_key_max_value",
            "low_value_max_value", "axis_key", "axis_value", "split_type")})

    def _build_masks(self) -> None:
        scores = get_scores_from_csv(self.model_name)
        if scores is None:
            if not self.num_layers:
                raise ValueError(f"no head-score table for {self.model_name!r}; pass num_layers "
                                 "to use a synthetic table")
            scores = synthetic_scores(int(self.num_layers), 1)
        self.head_scores = scores
        self.head_scores_mask = head_low_mask(scores, self.hybrid_ratio)
        self.layer_scores_mask = layer_low_mask(scores.shape[0])

    def update_params(self, **kwargs: Any) -> None:
        old = (self.hybrid_ratio, self.model_name)
        for k, v in kwargs.items():
            if hasattr(self, k) and v is not None:
                setattr(self, k, v)
        self.validate()
        if (self.hybrid_ratio, self.model_name) != old:
            self._build_masks()

    def _head_mask(self, layer_id: int, num_heads: int) -> torch.Tensor:
        m = self.head_scores_mask
        if m.shape[1] == 1 and num_heads > 1:
            m = m.expand(m.shape[0], num_heads)
        m = slice_for_tp(m, num_heads, self.tp_rank, self.tensor_parallel_size)
        return m[min(layer_id, m.shape[0] - 1)]

    def _layer_low(self, layer_id: int) -> bool:
        return bool(self.layer_scores_mask[min(layer_id, self.layer_scores_mask.shape[0] - 1)])

    def _split(self, layer_id: int, x: torch.Tensor):
        if self.split_type == "head":
            m = self._head_mask(layer_id, x.shape[2]).to(x.device)
            return x[:, :, m, :], x[:, :, ~m, :]
        empty = torch.zeros(0, dtype=x.dtype, device=x.device)
        return (x, empty) if self._layer_low(layer_id) else (empty, x)

    def quantize(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any):
        keys, values = tensor[0], tensor[1]
        lk, hk = self._split(layer_id, keys)
        lv, hv = self._split(layer_id, values)
        hk, hkm = quantize(self.high_key_max_value, hk, self.axis_key)
        hv, hvm = quantize(self.high_value_max_value, hv, self.axis_value)
        lk, lkm = quantize(self.low_key_max_value, lk, self.axis_key)
        lv, lvm = quantize(self.low_value_max_value, lv, self.axis_value)
        if self.split_type == "head":
            k = torch.cat([lk, hk], dim=2)
            v = torch.cat([lv, hv], dim=2)
        else:
            k = lk if lk.numel() else hk
            v = lv if lv.numel() else hv
        return torch.stack([k, v], 0), {
            "high_key_meta": hkm, "high_value_meta": hvm, "low_key_meta": lkm,
            "low_value_meta": lvm, "original_dtype": str(tensor.dtype).replace("torch.", "")}

    def quantize_into(self, layer_id: int, tensor: torch.Tensor, out: torch.Tensor) -> dict:
        """:meth:`quantize` of one layer ``[2, blocks, block_size, heads,
        dim]`` written straight into ``out`` (uint8 ``[2, heads, blocks,
        block_size, dim]``: the quantized tensor in heads-outer order, LOW
        heads first), the codes cast to uint8 as they are stored; returns the
        metadata.  Same codes and metadata as ``quantize`` followed by
        ``permute(0, 3, 1, 2, 4)``, without the concatenation and stacking
        copies."""
        empty = {"min_val": None, "quant_scale": None,
                 "original_dtype": str(tensor.dtype).replace("torch.", ""),
                 "quant_dtype": "uint8"}
        meta = {"original_dtype": str(tensor.dtype).replace("torch.", "")}
        for kv, (x, hi_v, lo_v, axis, hi_k, lo_k) in enumerate((
                (tensor[0], self.high_key_max_value, self.low_key_max_value, self.axis_key,
                 "high_key_meta", "low_key_meta"),
                (tensor[1], self.high_value_max_value, self.low_value_max_value,
                 self.axis_value, "high_value_meta", "low_value_meta"))):
            low, high = self._split(layer_id, x)
            n_low = low.shape[2] if low.dim() == 4 else 0
            for part, levels, key, dst in ((low, lo_v, lo_k, out[kv, :n_low]),
                                           (high, hi_v, hi_k, out[kv, n_low:])):
                if part.numel() == 0:
                    meta[key] = dict(empty)
                    continue
                q, meta[key] = _levels(levels, part, axis)
                dst.copy_(q.permute(2, 0, 1, 3))
        return {k: meta[k] for k in ("high_key_meta", "high_value_meta", "low_key_meta",
                                     "low_value_meta", "original_dtype")}

    def dequantize_into(self, layer_id: int, tensor: torch.Tensor, meta_data: Any,
                        out: torch.Tensor) -> None:
        """:meth:`dequantize` of one layer's codes (``[2, blocks, block_size,
        heads, dim]``, LOW heads first) written into ``out`` (same shape, the
        original dtype): each part is dequantized with the same arithmetic
        and placed at its heads with one index copy, without the full-size
        temporary and the stacking copy."""
        for kv, (hi, lo) in enumerate((("high_key_meta", "low_key_meta"),
                                       ("high_value_meta", "low_value_meta"))):
            part, dst = tensor[kv], out[kv]
            if self.split_type == "head":
                m = self._head_mask(layer_id, part.shape[2]).cpu()
                nlow = int(m.sum())
                idx = torch.arange(m.numel())
                for codes, key, heads in ((part[:, :, :nlow], lo, idx[m]),
                                          (part[:, :, nlow:], hi, idx[~m])):
                    if codes.numel():
                        dst.index_copy_(2, heads.to(dst.device),
                                        dequantize(codes, meta_data[key]).to(dst.dtype))
            else:
                key = lo if self._layer_low(layer_id) else hi
                dst.copy_(dequantize(part, meta_data[key]))

    def dequantize(self, layer_id: int, tensor: torch.Tensor, meta_data: Any, **kwargs: Any):
        keys, values = tensor[0], tensor[1]
        out = []
        for part, hi, lo in ((keys, "high_key_meta", "low_key_meta"),
                             (values, "high_value_meta", "low_value_meta")):
            if self.split_type == "head":
                m = self._head_mask(layer_id, part.shape[2]).to(part.device)
                nlow = int(m.sum())
                low = dequantize(part[:, :, :nlow], meta_data[lo])
                high = dequantize(part[:, :, nlow:], meta_data[hi])
                full = torch.empty((*part.shape[:2], part.shape[2], part.shape[3]),
                                   dtype=low.dtype if low.numel() else high.dtype,
                                   device=part.device)
                full[:, :, m] = low
                full[:, :, ~m] = high
            else:
                full = dequantize(part, meta_data[lo] if self._layer_low(layer_id)
                                  else meta_data[hi])
            out.append(full)
        return torch.stack(out, 0)


def fused_compatible(qc: Optional[dict]) -> bool:
    """True when a quantizer config is expressible by the fused kernels
    (channel keys, token values, head or layer split)."""
    qc = qc or {}
    return qc.get("axis_key", "channel") == "channel" and qc.get("axis_value", "token") == "token"
