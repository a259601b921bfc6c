"""Generic Transform -> Quantizer -> Codec pipeline (PyTorch ops).

Runs any ordered subset of the three stages layer by layer, then one codec
call over the heads-outer buffer ``[L, 2, H, B, bs, D]`` (reference:
kvserve_v1/compression/compression_manager.py:77-757).  Requests above
500 MiB are processed in chunks of 8 layers to bound the peak memory; if the
codec fails the raw bytes are sent and the metadata says so
(``codec_skipped`` / ``codec_error``).

The fused kernels (``fused_manager.py``) cover the default mode and every
custom pipeline whose quantizer uses channel keys and token values; this
manager serves the remaining configurations and reproduces the reference
pipeline's numerics exactly (its quantizer computes in the KV dtype).
"""

from __future__ import annotations

import time
from typing import Optional

import torch

from kvserve_hpdps_b200.compression.config import CompressedKVData, CompressionConfig
from kvserve_hpdps_b200.utils.logger import get_logger

logger = get_logger(__name__)

CHUNK_THRESHOLD_BYTES = 500 * 1024 * 1024
CHUNK_LAYERS = 8


class CompressionManager:
    def __init__(self, config: CompressionConfig, transformer=None, quantizer=None, codec=None):
        self.config = config
        self.transformer = transformer(**(config.transformer_config or {})) if transformer else None
        self.quantizer = quantizer(**(config.quantizer_config or {})) if quantizer else None
        self.codec = codec(**(config.codec_config or {})) if codec else None
        if config.enabled and config.pipeline:
            for stage, obj in (("transformer", self.transformer), ("quantizer", self.quantizer),
                               ("codec", self.codec)):
                if stage in config.pipeline and obj is None:
                    raise ValueError(f"pipeline stage {stage} has no component")
        self._last_decompress_timing: Optional[dict] = None

    def update_config(self, config: Optional[CompressionConfig]) -> None:
        if config is None:
            return
        self.config = config
        if self.transformer is not None:
            self.transformer.update_params(**(config.transformer_config or {}))
        if self.quantizer is not None:
            self.quantizer.update_params(**(config.quantizer_config or {}))
        if self.codec is not None:
            self.codec.update_params(**(config.codec_config or {}))

    # ------------------------------------------------------------ compress
    def _forward_layer(self, layer_id: int, data: torch.Tensor, qparams: list):
        if "transformer" in self.config.pipeline:
            data = self.transformer.transform(layer_id, data)
        if "quantizer" in self.config.pipeline:
            data, qp = self.quantizer.quantize(layer_id, data)
            qparams.append(qp)
        return data.permute(0, 3, 1, 2, 4)

    def _encode(self, buf: torch.Tensor, meta: dict, layer_id: int, request_id: str) -> torch.Tensor:
        if "codec" in self.config.pipeline:
            try:
                out = self.codec.encode(layer_id, buf)
                meta["codec_applied"] = True
                return out
            except Exception as e:  # noqa: BLE001
                logger.error("codec failed for %s layer %d: %s", request_id, layer_id, e)
                meta["codec_skipped"] = True
                meta["codec_error"] = f"{type(e).__name__}: {e}"
        return buf.reshape(-1).view(torch.uint8).contiguous()

    def _compress_range(self, data: torch.Tensor, start: int, request_id: str, meta: dict):
        qparams: list = []
        if "quantizer" in self.config.pipeline and hasattr(self.quantizer, "quantize_into"):
            # codes land in the heads-outer buffer directly (no per-layer stack)
            L, _, B, bs, H, D = data.shape
            buf = torch.empty((L, 2, H, B, bs, D), dtype=torch.uint8, device=data.device)
            for i in range(L):
                x = data[i]
                if "transformer" in self.config.pipeline:
                    x = self.transformer.transform(start + i, x)
                qparams.append(self.quantizer.quantize_into(start + i, x, buf[i]))
        else:
            layers = [self._forward_layer(start + i, data[i], qparams)
                      for i in range(data.shape[0])]
            buf = torch.stack(layers, 0).contiguous()
        if qparams:
            meta["quantization_params"] = qparams
            meta["quantization_applied"] = True
        if "transformer" in self.config.pipeline:
            meta["transformer_applied"] = True
        meta["codec_shape"] = list(buf.shape)
        meta["codec_dtype"] = str(buf.dtype).replace("torch.", "")
        return self._encode(buf, meta, start + data.shape[0] - 1, request_id)

    def compress_all_layers(self, all_layers_data: torch.Tensor, request_id: str,
                            config: Optional[CompressionConfig] = None,
                            metadata: Optional[dict] = None) -> Optional[CompressedKVData]:
        self.update_config(config)
        if not self.config.enabled or not self.config.pipeline:
            return None
        if not isinstance(all_layers_data, torch.Tensor) or all_layers_data.dim() != 6:
            logger.error("expected a 6-D KV tensor")
            return None
        try:
            L = all_layers_data.shape[0]
            size = all_layers_data.numel() * all_layers_data.element_size()
            if size < self.config.min_compress_size:
                return None
            base = {"request_id": request_id,
                    "original_dtype": str(all_layers_data.dtype).replace("torch.", ""),
                    "original_size": size, "device": str(all_layers_data.device),
                    "num_layers": L, "backend": "generic", **(metadata or {})}
            if size > CHUNK_THRESHOLD_BYTES:
                chunks, metas, total = [], [], 0
                n_chunks = (L + CHUNK_LAYERS - 1) // CHUNK_LAYERS
                for c in range(n_chunks):
                    s, e = c * CHUNK_LAYERS, min(L, (c + 1) * CHUNK_LAYERS)
                    cm = dict(base, start_layer_id=s, num_layers=e - s, chunk_index=c,
                              total_chunks=n_chunks)
                    body = self._compress_range(all_layers_data[s:e], s, request_id, cm)
                    cm["compressed_size"] = body.numel()
                    total += body.numel()
                    chunks.append(body)
                    metas.append(cm)
                return CompressedKVData(request_id=request_id, layer_id=L - 1, metadata=dict(
                    base, is_chunked=True, num_chunks=n_chunks), original_size=size,
                    compressed_size=total, is_chunked=True, chunks=chunks, chunk_metadata=metas)
            meta = dict(base, start_layer_id=0)
            t0 = time.monotonic()
            body = self._compress_range(all_layers_data, 0, request_id, meta)
            meta["t_quant_ms"] = (time.monotonic() - t0) * 1e3
            meta["compressed_size"] = body.numel()
            return CompressedKVData(request_id=request_id, layer_id=L - 1, compressed_tensor=body,
                                    metadata=meta, original_size=size,
                                    compressed_size=body.numel())
        except Exception as e:  # noqa: BLE001
            logger.error("compression failed for %s: %s", request_id, e)
            return None

    # ---------------------------------------------------------- decompress
    def _decode(self, body: torch.Tensor, meta: dict, layer_id: int) -> torch.Tensor:
        dtype, shape = meta.get("codec_dtype"), meta.get("codec_shape")
        if "codec" in self.config.pipeline and meta.get("codec_applied"):
            return self.codec.decode(layer_id, body, dtype, shape, meta.get("device", "cuda"))
        return body.view(getattr(torch, dtype)).reshape(shape)

    def _decompress_range(self, body: torch.Tensor, meta: dict) -> torch.Tensor:
        start = int(meta.get("start_layer_id", 0))
        cur = self._decode(body, meta, start)
        L = cur.shape[0]
        target = getattr(torch, meta.get("original_dtype", "bfloat16"))
        out = torch.empty((L, cur.shape[1], cur.shape[3], cur.shape[4], cur.shape[2],
                           cur.shape[5]), dtype=target, device=cur.device)
        direct = "quantizer" in self.config.pipeline and hasattr(self.quantizer, "dequantize_into")
        for i in range(L):
            x = cur[i].permute(0, 2, 3, 1, 4)
            if direct:
                # dequantized parts land in the output layer directly
                self.quantizer.dequantize_into(start + i, x, meta["quantization_params"][i],
                                               out[i])
                if "transformer" in self.config.pipeline:
                    out[i].copy_(self.transformer.inverse(start + i, out[i]).to(target))
                continue
            if "quantizer" in self.config.pipeline:
                x = self.quantizer.dequantize(start + i, x, meta["quantization_params"][i])
            if "transformer" in self.config.pipeline:
                x = self.transformer.inverse(start + i, x)
            out[i].copy_(x.to(target))
        return out

    def decompress_all_layers(self, compressed: CompressedKVData,
                              config: Optional[CompressionConfig] = None):
        self.update_config(config)
        if not self.config.enabled or not self.config.pipeline:
            return None
        try:
            t0 = time.monotonic()
            if compressed.is_chunked:
                return [self._decompress_range(c, m) for c, m in
                        zip(compressed.chunks, compressed.chunk_metadata)]
            out = self._decompress_range(compressed.compressed_tensor, compressed.metadata)
            self._last_decompress_timing = {"t_codec_decode_ms": 0.0,
                                            "t_dequant_ms": (time.monotonic() - t0) * 1e3}
            return out
        except Exception as e:  # noqa: BLE001
            logger.error("decompression failed for %s: %s", getattr(compressed, "request_id", None), e)
            return None
