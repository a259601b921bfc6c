"""Compression specs, defaults and the compressed-payload record.

Spec forms accepted in ``kv_connector_extra_config["compression"]``
(reference: kvserve_v1/compression/manager.py:54-120, README.md:110-176):

* ``None``: raw transfer, no compression;
* ``"default"``: the fused producer path (Hadamard + hybrid min-max quantizer
  + lossless codec) with ``DEFAULT_COMPRESSION_CONFIG``;
* a custom dict ``{"enabled", "pipeline", "transformer_config",
  "quantizer_config", "codec_config", "min_compress_size", ...}``;
* a controller dict ``{"mode": "controller", "library_path", ...}``.

``DEFAULT_COMPRESSION_CONFIG`` holds the same values as the reference's
(kvserve_v1/compression/compression_manager.py:16-36) so a profile tuned for
one builds the same quantizer in the other.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field
from typing import Any, Optional

import torch

DEFAULT_COMPRESSION_CONFIG: dict[str, Any] = {
    "enabled": True,
    "pipeline": ["quantizer", "codec"],
    "quantizer_config": {
        "model_name": "Llama-3.1-8B-Instruct",
        "hybrid_ratio": 0.8,
        "high_key_max_value": 12,
        "high_value_max_value": 8,
        "low_key_max_value": 6,
        "low_value_max_value": 4,
        "axis_key": "channel",
        "axis_value": "token",
        "split_type": "head",
    },
    "codec_config": {
        "codec_type": "nvcomp",
        "nvcomp_algorithm": "ANS",
        "data_type": "|u1",
    },
    "min_compress_size": 1024,
}

# Seed of the Rademacher signs in default mode (reference manager.py:159).
DEFAULT_HADAMARD_SEED = 0x3333

# Quantizer defaults when a key is missing from a custom quantizer_config
# (reference kvserve_quantizer.py:42-52).
QUANTIZER_DEFAULTS: dict[str, Any] = {
    "model_name": "Llama-3.1-8B-Instruct",
    "hybrid_ratio": 0.3,
    "high_key_max_value": 16,
    "high_value_max_value": 16,
    "low_key_max_value": 12,
    "low_value_max_value": 12,
    "axis_key": "channel",
    "axis_value": "token",
    "split_type": "head",
}

# Defaults the reference's fused op uses when built from a partial config
# (reference tilelang_manager.py:88-103).
FUSED_QUANTIZER_DEFAULTS: dict[str, Any] = {
    "hybrid_ratio": 0.5,
    "high_key_max_value": 12,
    "high_value_max_value": 8,
    "low_key_max_value": 6,
    "low_value_max_value": 4,
    "axis_key": "channel",
    "axis_value": "token",
    "split_type": "head",
}

VALID_PIPELINE_STAGES = ("transformer", "quantizer", "codec")


def get_default_compression_config() -> dict[str, Any]:
    """A deep copy of the default spec."""
    return copy.deepcopy(DEFAULT_COMPRESSION_CONFIG)


def validate_quantizer_config(qc: dict[str, Any]) -> None:
    """Raise ValueError on an invalid quantizer config (reference bounds:
    kvserve_quantizer.py:105-141)."""
    hr = float(qc.get("hybrid_ratio", 0.0))
    if not 0.0 <= hr <= 1.0:
        raise ValueError(f"hybrid_ratio must be in [0, 1], got {hr}")
    for key in ("low_key_max_value", "low_value_max_value",
                "high_key_max_value", "high_value_max_value"):
        v = qc.get(key)
        if v is None:
            continue
        if not 0 < float(v) < 255:
            raise ValueError(f"{key} must be in (0, 255), got {v}")
    for lo, hi in (("low_key_max_value", "high_key_max_value"),
                   ("low_value_max_value", "high_value_max_value")):
        if qc.get(lo) is not None and qc.get(hi) is not None and \
                float(qc[lo]) > float(qc[hi]):
            raise ValueError(f"{lo} must be <= {hi}")
    for key in ("axis_key", "axis_value"):
        if key in qc and qc[key] not in ("channel", "token", "tensor"):
            raise ValueError(f"{key} must be channel|token|tensor, got {qc[key]}")
    if "split_type" in qc and qc["split_type"] not in ("head", "layer"):
        raise ValueError(f"split_type must be head|layer, got {qc['split_type']}")


def validate_spec(spec: Any) -> None:
    """Validate a compression spec (None | "default" | dict)."""
    if spec is None or spec == "default":
        return
    if not isinstance(spec, dict):
        raise ValueError(f"compression spec must be None, 'default' or a dict, "
                         f"got {type(spec).__name__}")
    if spec.get("mode") == "controller":
        if "library_path" not in spec:
            raise ValueError("controller mode requires library_path")
        return
    for stage in spec.get("pipeline", []) or []:
        if stage not in VALID_PIPELINE_STAGES:
            raise ValueError(f"unknown pipeline stage {stage!r}")
    from kvserve_hpdps_b200.compression.components import custom_impls, resolve_component
    custom = custom_impls(spec)
    for kind, impl in custom.items():  # user components: resolvable, their configs their own
        resolve_component(kind, impl)
    if spec.get("quantizer_config") and "quantizer" not in custom:
        validate_quantizer_config(spec["quantizer_config"])
    cc = spec.get("codec_config")
    if cc and "codec" in (spec.get("pipeline") or []) and "codec" not in custom:
        # raises with the nvCOMP-name mapping for an unknown coder
        from kvserve_hpdps_b200.compression.codec import resolve_codec
        resolve_codec(cc.get("codec_type"), cc.get("nvcomp_algorithm"))
    overlap = spec.get("overlap", "off")
    if overlap not in ("off", "tq", "full", "stream"):
        raise ValueError(f"overlap must be off|tq|full|stream, got {overlap!r}")


@dataclass
class CompressionConfig:
    """Parsed generic pipeline config (reference compression_manager.py:44-58)."""
    enabled: bool = False
    transformer_config: Optional[dict[str, Any]] = None
    quantizer_config: Optional[dict[str, Any]] = None
    codec_config: Optional[dict[str, Any]] = None
    pipeline: Optional[list[str]] = None
    min_compress_size: int = 0


@dataclass
class CompressedKVData:
    """A compressed request (or layer group) before wire packing.

    Field names and meanings follow the reference record
    (kvserve_v1/compression/compression_manager.py:61-75) because the wire
    envelope serialises them by name.
    """
    request_id: str
    layer_id: int
    compressed_tensor: Optional[torch.Tensor] = None
    metadata: dict[str, Any] = field(default_factory=dict)
    original_size: int = 0
    compressed_size: int = 0
    is_chunked: bool = False
    chunks: Optional[list[torch.Tensor]] = None
    chunk_metadata: Optional[list[dict[str, Any]]] = None
