"""Environment-gated JSONL statistics and timeline markers.

The keys and the environment variables are those of the reference so that its
analysis scripts keep working:

* ``KVSERVE_COMPRESSION_STATS_PATH``: one row per compressed send
  (kvserve_v1/connector/compressed_kv_connector.py:57-87);
* ``KVSERVE_DECODE_STATS_PATH``: one row per decompression (:90-114);
* ``KVSERVE_TRANSFER_STATS_PATH``: one row per completed transfer
  (kvserve_v1/transport/nccl_transport.py:287-302);
* ``KVSERVE_TIMELINE_PATH``: ``"<tag> <epoch>"`` markers (:131-143).

Writers may add fields next to the reference keys (the transports add
``transport``); readers that only know the reference keys ignore them.

:func:`summarize` joins the three files into the figures the reference's
test drivers print: the mean per-row compression ratio
(tests/test_kvserve.py:420-458) and the median compress, communication and
decompress times with their serial sum ``xfer_path`` and the overlapped sum
``xfer_if_overlap`` (compress + comm, decompress hidden behind decode)
(scripts/xnode/run_cross_node.sh:273-308).  ``python -m
kvserve_hpdps_b200.utils.stats --compression c.jsonl --decode d.jsonl
--transfer t.jsonl`` prints it as one JSON object.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from typing import Any, Iterable, Optional

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


def read_rows(path: Optional[str]) -> list[dict[str, Any]]:
    """The JSON objects of a JSONL file; blank or malformed lines (a row cut
    off by a killed writer) are skipped, a missing file reads as empty."""
    if not path or not os.path.exists(path):
        return []
    rows = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            try:
                row = json.loads(line)
            except ValueError:
                continue
            if isinstance(row, dict):
                rows.append(row)
    return rows


def _numbers(rows: Iterable[dict], key: str) -> list[float]:
    return [float(r[key]) for r in rows
            if isinstance(r.get(key), (int, float)) and not isinstance(r.get(key), bool)]


def _median(rows: Iterable[dict], key: str) -> Optional[float]:
    vals = _numbers(rows, key)
    return statistics.median(vals) if vals else None


def summarize(compression: Optional[str] = None, decode: Optional[str] = None,
              transfer: Optional[str] = None) -> dict[str, Any]:
    """Summary of the stats files (any may be absent).

    ``avg_compression_ratio`` is the mean over rows of
    ``original_bytes / compressed_bytes``; ``aggregate_compression_ratio`` is
    the ratio of the byte sums.  Time fields are medians in ms; ``comm_ms``
    is the median ``transfer_ms`` and ``comm_mb`` the median transferred MB.
    ``xfer_path_ms`` = compress + comm + decompress, ``xfer_if_overlap_ms`` =
    compress + comm (absent parts count as 0, as in the reference table)."""
    c_rows = read_rows(compression)
    d_rows = read_rows(decode)
    t_rows = read_rows(transfer)
    ratios, orig, comp = [], 0, 0
    for r in c_rows:
        o, c = r.get("original_bytes"), r.get("compressed_bytes")
        if isinstance(o, (int, float)) and isinstance(c, (int, float)) and o > 0 and c > 0:
            ratios.append(o / c)
            orig += o
            comp += c
    out: dict[str, Any] = {
        "compression_rows": len(c_rows), "decode_rows": len(d_rows),
        "transfer_rows": len(t_rows),
        "avg_compression_ratio": sum(ratios) / len(ratios) if ratios else None,
        "aggregate_compression_ratio": orig / comp if comp else None,
    }
    for key in ("compress_ms", "quant_ms", "codec_ms", "prefill_span_ms"):
        out[key] = _median(c_rows, key)
    for key in ("decompress_ms", "codec_decode_ms", "dequant_ms"):
        out[key] = _median(d_rows, key)
    out["comm_ms"] = _median(t_rows, "transfer_ms")
    mb = _median(t_rows, "bytes")
    out["comm_mb"] = mb / 1e6 if mb is not None else None
    transports = sorted({str(r["transport"]) for r in t_rows if "transport" in r})
    out["transports"] = transports
    c = out["compress_ms"] or 0.0
    m = out["comm_ms"] or 0.0
    d = out["decompress_ms"] or 0.0
    out["xfer_path_ms"] = c + m + d
    out["xfer_if_overlap_ms"] = c + m
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="summarize KVServe JSONL stats files")
    ap.add_argument("--compression", default=os.environ.get("KVSERVE_COMPRESSION_STATS_PATH"))
    ap.add_argument("--decode", default=os.environ.get("KVSERVE_DECODE_STATS_PATH"))
    ap.add_argument("--transfer", default=os.environ.get("KVSERVE_TRANSFER_STATS_PATH"))
    args = ap.parse_args(argv)
    json.dump(summarize(args.compression, args.decode, args.transfer), sys.stdout,
              sort_keys=True)
    sys.stdout.write("\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
