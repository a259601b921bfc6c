"""Op-level API of the reference's fused Hadamard + quantization operator
(kvserve_v1/tilelang_ops/kv_hadamard_quant.py:37-66 ``make_rademacher_signs``,
``KVHadamardQuantOp``), served by this package's sm_100a kernels.

* ``compress_v3`` / ``decompress_v3`` (kv_hadamard_quant.py:1307-1480): one
  dense layer ``[2, blocks, block_size, heads, head_dim]`` bf16; keys are
  quantized per (head, channel) over all tokens, values per (token, group
  of heads with the same level count); the hybrid plan comes from the head
  scores at ``hybrid_ratio``.  The transform, statistics and quantization
  run in the fused tcgen05 kernels (the layer is addressed as a paged cache
  whose block table is the identity); ``decompress_v3`` runs the fused
  dequantize + inverse-transform kernel.  Codes are returned one byte per
  value in the input layout, metadata in the reference's dictionary form
  (``key_meta`` min/scale per (head, channel); ``value_meta`` per group,
  keyed by the group's level count, with ``head_idx`` and per-row
  min/scale).  Metadata travels as fp16, as on this package's wire.
* ``compress`` / ``decompress`` (kv_hadamard_quant.py:380-470, 1366-1408):
  the older per-(token, head) form, ``quant_type`` ``"absmax"`` (symmetric,
  ``q = trunc(clamp(y * m / (absmax + 1e-8), -m, m) + m)``, dequantized as
  ``(q - m) / m * absmax``) or ``"minmax"`` (``scale = max(max - min, 1e-5) / m``,
  ``q = clamp(floor((y - min) / scale + 0.5), 0, m)``), where ``m`` is the
  head's level count and ``y`` the fp32 transform of the fp16-rounded input.
  It is not on any serving path here and runs as PyTorch ops on the device.
"""

from __future__ import annotations

from typing import Optional

import torch

from kvserve_hpdps_b200.compression.signs import fwht_fp32, rademacher_signs

REFERENCE_DEFAULT_SEED = 0xC0FEBABE


def make_rademacher_signs(layer_id: int, num_heads: int, head_dim: int,
                          base_seed: int = REFERENCE_DEFAULT_SEED, device="cuda",
                          dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """[num_heads, head_dim] of +-1 seeded ``base_seed ^ (layer << 16) ^ head``."""
    return rademacher_signs(layer_id, num_heads, head_dim, base_seed).to(device=device,
                                                                           dtype=dtype)


class KVHadamardQuantOp:
    def __init__(self, num_heads: int = 8, head_dim: int = 128,
                 base_seed: int = REFERENCE_DEFAULT_SEED, dtype: torch.dtype = torch.bfloat16,
                 quant_type: str = "absmax", **kwargs):
        from kvserve_hpdps_b200.compression.fused_manager import FusedCompressionManager
        if quant_type not in ("absmax", "minmax"):
            raise ValueError(f"Unsupported quant_type: {quant_type}")
        self.num_heads = int(num_heads)
        self.head_dim = int(head_dim)
        self.base_seed = int(base_seed)
        self.dtype = dtype
        self.quant_type = quant_type
        self.model_name = kwargs.get("model_name", "Llama-3.1-8B-Instruct")
        self.hybrid_ratio = float(kwargs.get("hybrid_ratio", 0.3))
        self.high_key_max_value = float(kwargs.get("high_key_max_value", 16.0))
        self.high_value_max_value = float(kwargs.get("high_value_max_value", 16.0))
        self.low_key_max_value = float(kwargs.get("low_key_max_value", 12.0))
        self.low_value_max_value = float(kwargs.get("low_value_max_value", 12.0))
        self.split_type = kwargs.get("split_type", "head")
        qc = {"model_name": self.model_name, "hybrid_ratio": self.hybrid_ratio,
              "high_key_max_value": self.high_key_max_value,
              "high_value_max_value": self.high_value_max_value,
              "low_key_max_value": self.low_key_max_value,
              "low_value_max_value": self.low_value_max_value, "split_type": self.split_type}
        # byte codes, no entropy coder: compress_v3 hands codes to the caller
        self._mgr = FusedCompressionManager(self.num_heads, self.head_dim, qc,
                                            {"codec_type": "none"}, base_seed=self.base_seed,
                                            num_layers=kwargs.get("num_layers"))
        self._signs: dict[tuple, torch.Tensor] = {}

    # ------------------------------------------------------------ helpers
    def _get_signs(self, layer_id: int, device) -> torch.Tensor:
        key = (int(layer_id), str(device))
        if key not in self._signs:
            self._signs[key] = make_rademacher_signs(layer_id, self.num_heads, self.head_dim,
                                                     self.base_seed, device, torch.float32)
        return self._signs[key]

    def max_vals(self, layer_id: int, is_key: bool, device) -> torch.Tensor:
        """Level count per head of a layer (the hybrid plan)."""
        h = self._mgr.hybrid
        v = h.key_levels_for(layer_id) if is_key else h.value_levels_for(layer_id)
        return torch.as_tensor(v, dtype=torch.float32).to(device)

    # -------------------------------------------------------- v3 (default)
    def compress_v3(self, kv_layer: torch.Tensor, layer_id: int, axis_key: str = "channel",
                    axis_value: str = "token"):
        if axis_key != "channel" or axis_value != "token":
            raise ValueError("compress_v3 quantizes keys per channel and values per token")
        if kv_layer.dim() != 5 or kv_layer.shape[0] != 2:
            raise ValueError(f"expected [2, blocks, block_size, heads, dim], got "
                             f"{tuple(kv_layer.shape)}")
        if not kv_layer.is_cuda or kv_layer.dtype != torch.bfloat16:
            raise ValueError("compress_v3 needs a bf16 CUDA tensor")
        _, B, bs, H, D = kv_layer.shape
        codes, canon = self._mgr.compress_quant_layer(kv_layer, layer_id)
        q = codes.view(2, H, B, bs, D).permute(0, 2, 3, 1, 4).contiguous()
        kmv = self.max_vals(layer_id, True, kv_layer.device)
        vmv = self.max_vals(layer_id, False, kv_layer.device)
        groups = {}
        for g in canon["value_meta"]["per_group_list"]:
            lev = float(vmv[int(g["head_idx"][0])])
            groups[lev] = {"head_idx": g["head_idx"], "min_val": g["min_val"],
                           "quant_scale": g["quant_scale"]}
        value_meta = {"per_group_meta": groups}
        return q, {"key_meta": canon["key_meta"], "value_meta": value_meta,
                   "key_max_vals": kmv, "value_max_vals": vmv}

    def decompress_v3(self, q_kv: torch.Tensor, metadata: dict, layer_id: int) -> torch.Tensor:
        _, B, bs, H, D = q_kv.shape
        km = metadata["key_meta"]
        vm = metadata["value_meta"]
        if "per_group_meta" in vm:
            groups = [{"head_idx": g["head_idx"], "min_val": g["min_val"],
                       "quant_scale": g["quant_scale"]} for g in vm["per_group_meta"].values()]
        elif "per_group_list" in vm:
            groups = list(vm["per_group_list"])
        else:  # one group over every head
            groups = [{"head_idx": torch.arange(H), "min_val": vm["min_val"],
                       "quant_scale": vm["quant_scale"]}]
        dev = q_kv.device
        canon = {"key_meta": {"min_val": km["min_val"].to(dev), "quant_scale":
                              km["quant_scale"].to(dev), "axis": "channel"},
                 "value_meta": {"per_group_list": [
                     {"head_idx": g["head_idx"].to(torch.int64).cpu(),
                      "min_val": g["min_val"].to(dev).reshape(-1, 1, 1),
                      "quant_scale": g["quant_scale"].to(dev).reshape(-1, 1, 1)}
                     for g in groups]}}
        codes = q_kv.permute(0, 3, 1, 2, 4).contiguous().view(-1)
        out = torch.empty((1, 2, B, bs, H, D), dtype=torch.bfloat16, device=dev)
        self._mgr._dequant_dense(codes, [canon], [layer_id], out, self._mgr.base_seed)
        return out[0].to(self.dtype)

    # --------------------------------------------------- per-row (legacy)
    def _transform(self, kv: torch.Tensor, layer_id: int) -> torch.Tensor:
        s = self._get_signs(layer_id, kv.device).view(1, self.num_heads, self.head_dim)
        x = kv.reshape(-1, self.num_heads, self.head_dim).to(torch.float16).float()
        return fwht_fp32(x * s)

    def compress(self, kv: torch.Tensor, layer_id: int, is_key: bool = True,
                 max_val: Optional[float] = None):
        if kv.dtype != torch.bfloat16:
            raise ValueError("compress needs a bf16 tensor")
        nb, bs, H, D = kv.shape
        y = self._transform(kv, layer_id)  # [rows, H, D] fp32
        m = (torch.full((H,), float(max_val), device=kv.device) if max_val is not None
             else self.max_vals(layer_id, is_key, kv.device)).view(1, H, 1)
        if self.quant_type == "absmax":
            s = y.abs().amax(-1, keepdim=True)
            q = (torch.maximum(torch.minimum(y * (m / (s + 1e-8)), m), -m) + m)
            q = q.to(torch.uint8)  # truncation of a non-negative value
            meta = {"scales": s.reshape(-1), "max_vals": m.reshape(-1)}
        else:
            lo, hi = y.amin(-1, keepdim=True), y.amax(-1, keepdim=True)
            scale = torch.clamp(hi - lo, min=1e-5) / m
            q = torch.floor((y - lo) * (1.0 / scale) + 0.5).clamp(min=0).minimum(m)
            q = q.to(torch.uint8)
            meta = {"scales": scale.reshape(-1), "mins": lo.reshape(-1),
                    "max_vals": m.reshape(-1)}
        return q.reshape(nb, bs, H, D), meta

    def decompress(self, q_kv: torch.Tensor, metadata: dict, layer_id: int,
                   max_val: Optional[float] = None) -> torch.Tensor:
        nb, bs, H, D = q_kv.shape
        dev = q_kv.device
        q = q_kv.float().view(nb, bs, H, D)
        s = metadata["scales"].to(dev).view(nb, bs, H, 1)
        m = metadata["max_vals"].to(dev).view(1, 1, H, 1)
        if self.quant_type == "absmax":
            y = (q - m) / m * s
        else:
            y = q * s + metadata["mins"].to(dev).view(nb, bs, H, 1)
        y = y.to(self.dtype).float()
        x = fwht_fp32(y) * self._get_signs(layer_id, dev).view(1, 1, H, D)
        return x.to(self.dtype)

    def __repr__(self) -> str:
        return (f"KVHadamardQuantOp(heads={self.num_heads}, head_dim={self.head_dim}, "
                f"quant_type={self.quant_type}, hybrid_ratio={self.hybrid_ratio})")


__all__ = ["KVHadamardQuantOp", "make_rademacher_signs", "REFERENCE_DEFAULT_SEED"]
