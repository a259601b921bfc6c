"""Environment-gated JSONL statistics and timeline markers.

The keys and the environment variables are those of the reference so that its
analysis scripts keep working:

* ``KVSERVE_COMPRESSION_STATS_PATH``: one row per compressed send
  (kvserve_v1/connector/compressed_kv_connector.py:57-87);
* ``KVSERVE_DECODE_STATS_PATH``: one row per decompression (:90-114);
* ``KVSERVE_TRANSFER_STATS_PATH``: one row per completed transfer
  (kvserve_v1/transport/nccl_transport.py:287-302);
* ``KVSERVE_TIMELINE_PATH``: ``"<tag> <epoch>"`` markers (:131-143).

Rows written here add device-timed fields (``*_device_ms``) next to the
reference keys; readers that only know the reference keys ignore them.
"""

from __future__ import annotations

import json
import os
import threading
import time
from typing import Any

_lock = threading.Lock()


def _append(path: str | None, row: dict[str, Any]) -> None:
    if not path:
        return
    try:
        line = json.dumps(row, sort_keys=True) + "\n"
        with _lock, open(path, "a") as f:
            f.write(line)
    except OSError:
        pass


def write_compression_stats(request_id: str, transfer_id: str,
                            original_bytes: int, compressed_bytes: int,
                            compress_ms: float = 0.0, quant_ms: float = 0.0,
                            codec_ms: float = 0.0, prefill_span_ms: float = 0.0,
                            **extra: Any) -> None:
    if original_bytes <= 0 or compressed_bytes <= 0:
        return
    row = {"request_id": request_id, "transfer_id": transfer_id,
           "original_bytes": int(original_bytes),
           "compressed_bytes": int(compressed_bytes),
           "compress_ms": float(compress_ms), "quant_ms": float(quant_ms),
           "codec_ms": float(codec_ms),
           "prefill_span_ms": float(prefill_span_ms)}
    row.update(extra)
    _append(os.environ.get("KVSERVE_COMPRESSION_STATS_PATH"), row)


def write_decode_stats(request_id: str, transfer_id: str, decompress_ms: float,
                       codec_decode_ms: float = 0.0, dequant_ms: float = 0.0,
                       **extra: Any) -> None:
    row = {"request_id": request_id, "transfer_id": transfer_id,
           "decompress_ms": float(decompress_ms),
           "codec_decode_ms": float(codec_decode_ms),
           "dequant_ms": float(dequant_ms)}
    row.update(extra)
    _append(os.environ.get("KVSERVE_DECODE_STATS_PATH"), row)


def write_transfer_stats(request_id: str, transfer_ms: float, nbytes: int,
                         **extra: Any) -> None:
    row = {"request_id": request_id, "transfer_ms": float(transfer_ms),
           "bytes": int(nbytes)}
    row.update(extra)
    _append(os.environ.get("KVSERVE_TRANSFER_STATS_PATH"), row)


def timeline(tag: str) -> None:
    path = os.environ.get("KVSERVE_TIMELINE_PATH")
    if not path:
        return
    try:
        with _lock, open(path, "a") as f:
            f.write("%s %.4f\n" % (tag, time.time()))
    except OSError:
        pass
