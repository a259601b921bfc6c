"""Transform stage of the generic pipeline: randomized Hadamard.

Reference semantics (kvserve_v1/compression/transformer/*): per (layer,
head) Rademacher signs seeded with ``seed ^ (layer << 16) ^ head``; forward
``FWHT(x * s) / sqrt(D)``, inverse ``FWHT(y) / sqrt(D) * s``; head
dimensions that are not powers of two are transformed per power-of-two
chunk.  The output keeps the input dtype.  The generic pipeline is only used
for configurations the fused kernels do not cover; the transform runs as an
fp32 product with the +-1 matrix on the tensor's device.
"""

from __future__ import annotations

from typing import Any

import torch

from kvserve_hpdps_b200.compression.components import Transformer
from kvserve_hpdps_b200.compression.signs import fwht_fp32, rademacher_signs


class HadamardTransform:
    def __init__(self, base_seed: int = 0xC0FEBABE):
        self.base_seed = base_seed
        self._signs: dict[tuple, torch.Tensor] = {}

    def signs(self, layer_id: int, num_heads: int, head_dim: int, device, dtype) -> torch.Tensor:
        key = (layer_id, num_heads, head_dim, str(device), dtype)
        if key not in self._signs:
            s = rademacher_signs(layer_id, num_heads, head_dim, self.base_seed)
            self._signs[key] = s.to(device=device, dtype=dtype).view(1, 1, num_heads, head_dim)
        return self._signs[key]

    # the reference's name (hadamard_func.py:105-159): [1, 1, heads, head_dim] +-1
    get_rademacher_signs = signs

    def transform(self, layer_id: int, x: torch.Tensor) -> torch.Tensor:
        s = self.signs(layer_id, x.shape[2], x.shape[3], x.device, x.dtype)
        return fwht_fp32(x * s).to(x.dtype)

    def inverse(self, layer_id: int, y: torch.Tensor) -> torch.Tensor:
        s = self.signs(layer_id, y.shape[2], y.shape[3], y.device, y.dtype)
        return fwht_fp32(y).to(y.dtype) * s


class KVServeTransformer(Transformer):
    """``transformer_config = {"transform_type": "hadamard", "seed": 0x3333}``."""

    def __init__(self, **kwargs: Any):
        self.transform_type = kwargs.get("transform_type", "hadamard")
        self.seed = kwargs.get("seed", 0x3333)
        self.validate()
        self.impl = HadamardTransform(self.seed)

    def validate(self) -> None:
        if self.transform_type != "hadamard":
            raise ValueError(f"invalid transform type {self.transform_type!r}")
        if self.seed is None:
            raise ValueError("seed is required")

    def update_params(self, **kwargs: Any) -> None:
        super().update_params(**kwargs)
        self.validate()
        self.impl = HadamardTransform(self.seed)

    def transform(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        out = torch.empty_like(tensor)
        out[0] = self.impl.transform(layer_id, tensor[0])
        out[1] = self.impl.transform(layer_id, tensor[1])
        return out

    def inverse(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        out = torch.empty_like(tensor)
        out[0] = self.impl.inverse(layer_id, tensor[0])
        out[1] = self.impl.inverse(layer_id, tensor[1])
        return out
