"""Wire envelope of a compressed payload: msgpack-safe metadata + tensors.

A :class:`CompressedKVData` is split into ``meta`` (plain Python values,
serialisable with msgpack), ``body_chunks`` (the coded bytes, split into
chunks of at most ``max_chunk_bytes``) and ``aux_tensors`` (every tensor found
under ``quantization_params``, replaced in ``meta`` by the placeholder
``["__kvserve_aux_tensor__", index]``).  Body modes: ``single``,
``byte_chunks`` (one tensor split into byte chunks) and ``manager_chunks``
(a chunked payload, one body per chunk).

The placeholder string, the meta keys and the body modes are those of the
reference envelope (kvserve_v1/compression/wire.py:16-131) so that both
ends agree on the message layout.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from kvserve_hpdps_b200.compression.config import CompressedKVData

AUX_PLACEHOLDER = "__kvserve_aux_tensor__"
DEFAULT_MAX_CHUNK_BYTES = 512 * 1024 * 1024


@dataclass
class CompressedWire:
    meta: dict[str, Any]
    body_chunks: list[torch.Tensor]
    aux_tensors: list[torch.Tensor]

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.body_chunks + self.aux_tensors)


def _spec(t: torch.Tensor) -> dict[str, Any]:
    return {"shape": list(t.shape), "dtype": str(t.dtype).replace("torch.", "")}


def _pack(obj: Any, aux: list[torch.Tensor]) -> Any:
    if isinstance(obj, torch.Tensor):
        aux.append(obj.contiguous())
        return [AUX_PLACEHOLDER, len(aux) - 1]
    if isinstance(obj, dict):
        return {k: _pack(v, aux) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return [_pack(v, aux) for v in obj]
    return obj


def _is_placeholder(obj: Any) -> bool:
    return isinstance(obj, list) and len(obj) == 2 and obj[0] == AUX_PLACEHOLDER


def _unpack(obj: Any, aux: list[torch.Tensor]) -> Any:
    if _is_placeholder(obj):
        return aux[int(obj[1])]
    if isinstance(obj, dict):
        return {k: _unpack(v, aux) for k, v in obj.items()}
    if isinstance(obj, list):
        return [_unpack(v, aux) for v in obj]
    return obj


def pack_metadata(meta: Any, aux: list[torch.Tensor]) -> Any:
    """Replace tensors under ``quantization_params`` by aux placeholders."""
    if not isinstance(meta, dict):
        return meta
    out = dict(meta)
    if "quantization_params" in out:
        out["quantization_params"] = _pack(out["quantization_params"], aux)
    return out


def unpack_metadata(meta: Any, aux: list[torch.Tensor]) -> Any:
    if isinstance(meta, dict) and "quantization_params" in meta:
        meta = dict(meta)
        meta["quantization_params"] = _unpack(meta["quantization_params"], aux)
    return meta


def assert_no_tensor(obj: Any) -> None:
    if isinstance(obj, torch.Tensor):
        raise TypeError("wire metadata still holds a tensor outside quantization_params")
    if isinstance(obj, dict):
        for v in obj.values():
            assert_no_tensor(v)
    elif isinstance(obj, (list, tuple)):
        for v in obj:
            assert_no_tensor(v)


def split_bytes(t: torch.Tensor, max_chunk_bytes: int) -> list[torch.Tensor]:
    if max_chunk_bytes <= 0:
        raise ValueError("max_chunk_bytes must be positive")
    b = t.contiguous().view(torch.uint8).reshape(-1)
    return [b[i:i + max_chunk_bytes] for i in range(0, b.numel(), max_chunk_bytes)] or [b]


def build_wire(compressed: CompressedKVData,
               max_chunk_bytes: int = DEFAULT_MAX_CHUNK_BYTES) -> CompressedWire:
    aux: list[torch.Tensor] = []
    if compressed.is_chunked:
        if not compressed.chunks or not compressed.chunk_metadata:
            raise ValueError("chunked payload without chunks or chunk metadata")
        meta = {"is_chunked": True, "layer_id": compressed.layer_id,
                "original_size": compressed.original_size,
                "compressed_size": compressed.compressed_size,
                "metadata": pack_metadata(compressed.metadata, aux),
                "chunk_metadata": [pack_metadata(m, aux) for m in compressed.chunk_metadata],
                "body_mode": "manager_chunks"}
        assert_no_tensor(meta)
        return CompressedWire(meta, [c.contiguous() for c in compressed.chunks], aux)
    if compressed.compressed_tensor is None:
        raise ValueError("non-chunked payload without compressed_tensor")
    body = compressed.compressed_tensor.contiguous()
    nbytes = body.numel() * body.element_size()
    if nbytes > max_chunk_bytes:
        chunks, mode = split_bytes(body, max_chunk_bytes), "byte_chunks"
    else:
        chunks, mode = [body], "single"
    meta = {"is_chunked": False, "layer_id": compressed.layer_id,
            "original_size": compressed.original_size,
            "compressed_size": compressed.compressed_size,
            "metadata": pack_metadata(compressed.metadata, aux),
            "body_mode": mode, "body_spec": _spec(body)}
    assert_no_tensor(meta)
    return CompressedWire(meta, chunks, aux)


def restore_from_wire(wire: CompressedWire) -> CompressedKVData:
    meta = wire.meta
    inner = unpack_metadata(meta.get("metadata"), wire.aux_tensors)
    rid = str(inner.get("request_id", "unknown")) if isinstance(inner, dict) else "unknown"
    if meta.get("is_chunked"):
        return CompressedKVData(
            request_id=rid, layer_id=int(meta.get("layer_id", -1)), compressed_tensor=None,
            metadata=inner, original_size=int(meta.get("original_size", 0)),
            compressed_size=int(meta.get("compressed_size", 0)), is_chunked=True,
            chunks=list(wire.body_chunks),
            chunk_metadata=[unpack_metadata(m, wire.aux_tensors)
                            for m in meta.get("chunk_metadata", [])])
    if meta.get("body_mode") == "byte_chunks":
        raw = torch.cat([c.contiguous().view(torch.uint8).reshape(-1) for c in wire.body_chunks])
        spec = meta["body_spec"]
        body = raw.view(getattr(torch, spec["dtype"])).reshape(spec["shape"])
    else:
        body = wire.body_chunks[0]
    return CompressedKVData(request_id=rid, layer_id=int(meta.get("layer_id", -1)),
                            compressed_tensor=body, metadata=inner,
                            original_size=int(meta.get("original_size", 0)),
                            compressed_size=int(meta.get("compressed_size", 0)))
