"""Component interfaces of the Transform -> Quantizer -> Codec pipeline.

A new component subclasses one of these and is selected by name in the
pipeline (reference: kvserve_v1/compression/components.py:11-108).  Shapes:
per-layer KV tensors are ``[2, num_blocks, block_size, num_heads, head_dim]``;
codec inputs are uint8 (or any dtype, viewed as bytes).
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any, Optional

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


# ------------------------------------------------------------------ registry
# A pipeline spec names its own component classes with ``transformer_impl``,
# ``quantizer_impl`` or ``codec_impl``: a name registered here, or an import
# path ``package.module:Class`` (also ``package.module.Class``).  The
# reference documents the ``quantizer_impl`` key for user quantizers
# (kvserve_v1 examples/README.md:46-58) but its adapter never reads it
# (compression/manager.py:192-212); here all three stages take one.

_KINDS = {"transformer": ("transform", "inverse"), "quantizer": ("quantize", "dequantize"),
          "codec": ("encode", "decode")}
_REGISTRY: dict[str, dict[str, type]] = {k: {} for k in _KINDS}


def register_component(kind: str, name: str, cls: type) -> type:
    """Make ``cls`` selectable as ``<kind>_impl: name``.  Returns ``cls`` (so
    it also works as ``register_component("quantizer", "q", MyQ)`` after the
    class body)."""
    if kind not in _KINDS:
        raise ValueError(f"component kind must be one of {sorted(_KINDS)}, got {kind!r}")
    _check(kind, cls, name)
    _REGISTRY[kind][name] = cls
    return cls


def _check(kind: str, cls: Any, name: str) -> None:
    missing = [m for m in _KINDS[kind] if not callable(getattr(cls, m, None))]
    if missing:
        raise TypeError(f"{kind} component {name!r} lacks {missing}")


def resolve_component(kind: str, impl: Any) -> Optional[type]:
    """The class a ``<kind>_impl`` value names (None: the built-in one)."""
    if impl is None:
        return None
    if kind not in _KINDS:
        raise ValueError(f"component kind must be one of {sorted(_KINDS)}, got {kind!r}")
    if isinstance(impl, type):
        cls = impl
    elif not isinstance(impl, str) or not impl:
        raise ValueError(f"{kind}_impl must be a registered name or an import path, got {impl!r}")
    elif impl in _REGISTRY[kind]:
        cls = _REGISTRY[kind][impl]
    elif ":" in impl or "." in impl:
        import importlib
        mod_name, _, attr = impl.partition(":") if ":" in impl else impl.rpartition(".")
        try:
            cls = getattr(importlib.import_module(mod_name), attr)
        except (ImportError, AttributeError) as e:
            raise ValueError(f"{kind}_impl {impl!r} cannot be imported: {e}") from e
    else:
        raise ValueError(f"unknown {kind}_impl {impl!r}; registered: "
                         f"{sorted(_REGISTRY[kind]) or 'none'} (or give module:Class)")
    _check(kind, cls, str(impl))
    return cls


def custom_impls(cfg: Optional[dict]) -> dict[str, str]:
    """The stages of a spec that name their own component."""
    return {k: cfg[f"{k}_impl"] for k in _KINDS
            if isinstance(cfg, dict) and cfg.get(f"{k}_impl") is not None}
