"""Component interfaces of the Transform -> Quantizer -> Codec pipeline.

A new component subclasses one of these and is selected by name in the
pipeline (reference: kvserve_v1/compression/components.py:11-108).  Shapes:
per-layer KV tensors are ``[2, num_blocks, block_size, num_heads, head_dim]``;
codec inputs are uint8 (or any dtype, viewed as bytes).
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any

import torch


class Transformer(ABC):
    """Invertible per-layer transform applied before quantization."""

    @abstractmethod
    def transform(self, layer_id: int, tensor: torch.Tensor, **kwargs) -> torch.Tensor:
        ...

    @abstractmethod
    def inverse(self, layer_id: int, tensor: torch.Tensor, **kwargs) -> torch.Tensor:
        ...

    def update_params(self, **kwargs) -> None:
        for key, value in kwargs.items():
            if hasattr(self, key):
                setattr(self, key, value)


class Quantizer(ABC):
    """Lossy quantizer: returns (codes, params) and reverses with params."""

    @abstractmethod
    def quantize(self, layer_id: int, tensor: torch.Tensor, **kwargs) -> tuple[torch.Tensor, dict[str, Any]]:
        ...

    @abstractmethod
    def dequantize(self, layer_id: int, tensor: torch.Tensor, meta_data: Any, **kwargs) -> torch.Tensor:
        ...

    def update_params(self, **kwargs) -> None:
        for key, value in kwargs.items():
            if hasattr(self, key):
                setattr(self, key, value)


class Codec(ABC):
    """Lossless byte codec."""

    @abstractmethod
    def encode(self, layer_id: int, tensor: torch.Tensor, **kwargs) -> torch.Tensor:
        ...

    @abstractmethod
    def decode(self, layer_id: int, compressed_data: torch.Tensor, original_dtype: str,
               original_shape: list[int], device: str, **kwargs) -> torch.Tensor:
        ...

    def update_params(self, **kwargs) -> None:
        for key, value in kwargs.items():
            if hasattr(self, key):
                setattr(self, key, value)
