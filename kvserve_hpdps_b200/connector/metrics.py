"""KV-transfer statistics for vLLM's connector-stats logging and Prometheus.

vLLM collects a ``KVConnectorStats`` object from every worker after each
step (``get_kv_connector_stats``), aggregates them across workers, logs the
reduced figures at its logging interval and hands the raw data to the
connector's Prometheus metrics (``build_kv_connector_stats``,
``build_prom_metrics``).  The reference does not use these hooks; its
figures only reach the env-gated JSONL files (kvserve_v1/connector/
compressed_kv_connector.py:57-114), which this package writes as well.

Producer rows: one per message that left (original and wire bytes,
compression ms on the engine thread, transfer ms from the transport: the
device time from the message's first kernel to its last store on the ring
transport).  Consumer rows: decode ms per request, and counters of failed
sends and failed loads.  Data lives in plain lists so that the object
pickles from the worker to the logger process.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Any

try:  # vLLM is optional for importing this module (unit tests mock it)
    from vllm.distributed.kv_transfer.kv_connector.v1.metrics import (KVConnectorPromMetrics,
                                                                      KVConnectorStats)
except Exception:  # noqa: BLE001
    @dataclass
    class KVConnectorStats:  # type: ignore[no-redef]
        data: dict[str, Any] = field(default_factory=dict)

    class KVConnectorPromMetrics:  # type: ignore[no-redef]
        def __init__(self, vllm_config, metric_types, labelnames, per_engine_labelvalues):
            self._gauge_cls = next(v for k, v in metric_types.items() if k.__name__ == "Gauge")
            self._counter_cls = next(v for k, v in metric_types.items()
                                     if k.__name__ == "Counter")
            self._histogram_cls = next(v for k, v in metric_types.items()
                                       if k.__name__ == "Histogram")
            self._labelnames = labelnames
            self.per_engine_labelvalues = per_engine_labelvalues

SERIES = ("original_bytes", "wire_bytes", "compress_ms", "transfer_ms", "decode_ms",
          "failed_sends", "failed_loads")


def _percentile(xs: list, q: float) -> float:
    s = sorted(xs)
    if not s:
        return 0.0
    k = (len(s) - 1) * q
    lo = int(k)
    hi = min(lo + 1, len(s) - 1)
    return s[lo] + (s[hi] - s[lo]) * (k - lo)


@dataclass
class KVServeConnectorStats(KVConnectorStats):
    """Per-interval series of one worker, or of all workers once aggregated."""

    def __post_init__(self):
        self._lock = threading.Lock()
        for k in SERIES:
            self.data.setdefault(k, [])

    def __getstate__(self) -> dict:
        st = self.__dict__.copy()
        st.pop("_lock", None)
        return st

    def __setstate__(self, st: dict) -> None:
        self.__dict__.update(st)
        self._lock = threading.Lock()

    def reset(self) -> None:
        with self._lock:
            self.data = {k: [] for k in SERIES}

    # ---------------------------------------------------------- recording
    def record_sent(self, original_bytes: int, wire_bytes: int, compress_ms: float,
                    transfer_ms: float) -> None:
        """One message that left the producer (raw KV: original == wire)."""
        with self._lock:
            self.data["original_bytes"].append(int(original_bytes))
            self.data["wire_bytes"].append(int(wire_bytes))
            self.data["compress_ms"].append(float(compress_ms))
            self.data["transfer_ms"].append(float(transfer_ms))

    def record_decode(self, ms: float) -> None:
        with self._lock:
            self.data["decode_ms"].append(float(ms))

    def record_failed_send(self, n: int = 1) -> None:
        with self._lock:
            self.data["failed_sends"].extend([1] * int(n))

    def record_failed_load(self, n: int = 1) -> None:
        with self._lock:
            self.data["failed_loads"].extend([1] * int(n))

    def clone_and_reset(self) -> "KVServeConnectorStats":
        """The interval's data as a new object; this one starts over."""
        with self._lock:
            snap = {k: list(v) for k, v in self.data.items()}
            self.data = {k: [] for k in SERIES}
        return KVServeConnectorStats(data=snap)

    # ---------------------------------------------------------- vLLM API
    def is_empty(self) -> bool:
        return not any(self.data.get(k) for k in SERIES)

    def aggregate(self, other: "KVConnectorStats") -> "KVServeConnectorStats":
        if other is not None and not other.is_empty():
            with self._lock:
                for k in SERIES:
                    self.data.setdefault(k, []).extend(other.data.get(k, []))
        return self

    def reduce(self) -> dict[str, int | float]:
        d = self.data
        n = len(d["wire_bytes"])
        orig, wire = sum(d["original_bytes"]), sum(d["wire_bytes"])
        xfer_s = sum(d["transfer_ms"]) / 1e3
        mean = (lambda xs: round(sum(xs) / len(xs), 3) if xs else 0.0)
        return {
            "Num messages sent": n,
            "Compression ratio": round(orig / wire, 3) if wire else 0.0,
            "Avg MB per message (original)": round(orig / max(1, n) / 2**20, 3),
            "Avg compress time (ms)": mean(d["compress_ms"]),
            "Avg transfer time (ms)": mean(d["transfer_ms"]),
            "P90 transfer time (ms)": round(_percentile(d["transfer_ms"], 0.9), 3),
            "Throughput of original KV (MB/s)": round(orig / 2**20 / xfer_s, 3) if xfer_s else 0.0,
            "Num decoded": len(d["decode_ms"]),
            "Avg decode time (ms)": mean(d["decode_ms"]),
            "Num failed sends": len(d["failed_sends"]),
            "Num failed loads": len(d["failed_loads"]),
        }


class KVServePromMetrics(KVConnectorPromMetrics):
    """Prometheus series per engine: byte counters (original and on the
    wire), histograms of compress / transfer / decode time, failure
    counters."""

    def __init__(self, vllm_config, metric_types, labelnames, per_engine_labelvalues):
        super().__init__(vllm_config, metric_types, labelnames, per_engine_labelvalues)
        ms_buckets = [0.1, 0.25, 0.5, 1, 2.5, 5, 10, 25, 50, 100, 250, 1000]

        def per_engine(metric):
            return {i: metric.labels(*v) for i, v in per_engine_labelvalues.items()}

        self.original = per_engine(self._counter_cls(
            name="vllm:kvserve_original_bytes", documentation="KV bytes handed off, before "
            "compression", labelnames=labelnames))
        self.wire = per_engine(self._counter_cls(
            name="vllm:kvserve_wire_bytes", documentation="KV bytes that crossed the link",
            labelnames=labelnames))
        self.hist = {k: per_engine(self._histogram_cls(
            name=f"vllm:kvserve_{k}_seconds", documentation=doc, buckets=[b / 1e3 for b in
                                                                           ms_buckets],
            labelnames=labelnames)) for k, doc in (
                ("compress", "compression time per message"),
                ("transfer", "transfer time per message (device-timed on the ring)"),
                ("decode", "decode time per request"))}
        self.failed = {k: per_engine(self._counter_cls(
            name=f"vllm:kvserve_failed_{k}", documentation=f"failed {k}",
            labelnames=labelnames)) for k in ("sends", "loads")}

    def observe(self, transfer_stats_data: dict[str, Any], engine_idx: int = 0) -> None:
        d = transfer_stats_data or {}
        self.original[engine_idx].inc(sum(d.get("original_bytes", [])))
        self.wire[engine_idx].inc(sum(d.get("wire_bytes", [])))
        for key, series in (("compress", "compress_ms"), ("transfer", "transfer_ms"),
                            ("decode", "decode_ms")):
            for v in d.get(series, []):
                self.hist[key][engine_idx].observe(v / 1e3)
        for k in ("sends", "loads"):
            n = len(d.get(f"failed_{k}", []))
            if n:
                self.failed[k][engine_idx].inc(n)
