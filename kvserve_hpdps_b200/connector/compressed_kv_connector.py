"""CompressedKVConnector: vLLM V1 KV connector for prefill/decode disaggregation.

Load it with ``KVTransferConfig(kv_connector="CompressedKVConnector",
kv_connector_module_path="kvserve_hpdps_b200.connector.compressed_kv_connector",
kv_role="kv_producer"|"kv_consumer", kv_rank=0|1, kv_parallel_size=2,
kv_ip=<decode host>, kv_port=<base>, kv_connector_extra_config={"compression":
None | "default" | {...}})``.  ``transfer_id`` comes from
``SamplingParams(extra_args={"kv_transfer_params": {"transfer_id": ...}})``.
Public contract and scheduler logic follow the reference connector
(kvserve_v1/connector/compressed_kv_connector.py:189-1060).

Scheduler side (both roles): transfer ids are resolved from the request's
``kv_transfer_params`` (falling back to the request id); the producer defers
chunked prefills until the whole prompt's KV exists; the consumer claims
``len(prompt) - 1`` external tokens (one token is computed locally) and
loads the KV of newly scheduled and preemption-resumed requests.

Worker side:

* producer, ``overlap="off"`` (default): ``wait_for_save`` compresses every
  layer of every finished prefill with one batched set of fused launches per
  request, on the forward's stream (device ordering protects the blocks from
  reuse, no host sync), and sends one message per request;
* producer, ``overlap="stream"``: ``save_kv_layer`` compresses the layer for
  all requests of the step on a side stream (one grouped message per layer)
  while the next layers compute; ``wait_for_save`` makes the forward stream
  wait on the side stream;
* consumer, ``overlap="off"``: ``start_load_kv`` drains the transport, waits
  (bounded) for each scheduled request's message and decodes it straight
  into the registered paged caches at the consumer's block ids (fused
  dequantize + inverse transform + scatter); raw payloads are scattered with
  the block-copy kernel;
* consumer, ``overlap="stream"``: loading is layer-wise.  ``start_load_kv``
  decodes the layers that have arrived on a load stream and returns;
  ``wait_for_layer_load(l)`` waits on the host only for layer l's message
  headers and makes the forward stream wait on the device for layer l's
  decode, so the first layers' attention runs while later layers are still
  being pushed (the reference's ``wait_for_layer_load`` is a no-op,
  kvserve_v1/connector/compressed_kv_connector.py:570-571).  A grouped
  message (one layer of every request of the producer's step) is decoded
  once for all of its members scheduled in the step.

Transports: ``"p2p"`` (NVLink receive ring, producer kernels store into the
consumer's memory), ``"nccl"`` (reference protocol over a torch NCCL group)
or ``"auto"`` (p2p when both GPUs are visible to the producer, else nccl);
``kv_connector_extra_config["transport"]`` or ``KVSERVE_TRANSPORT`` selects.
"""

from __future__ import annotations

import os
import re
import threading
import time
from collections import defaultdict, deque
from contextlib import nullcontext
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any, Optional

import torch

from kvserve_hpdps_b200.compression.manager import (add_sentinel, is_compressed_layer_names,
                                                    strip_sentinel)
from kvserve_hpdps_b200.compression.wire import CompressedWire, build_wire, restore_from_wire
from kvserve_hpdps_b200.connector.metrics import KVServeConnectorStats, KVServePromMetrics
from kvserve_hpdps_b200.utils.kv_utils import (extract_kv_from_layer_by_blocks,
                                               inject_kv_into_layer_by_blocks, make_slot_mapping)
from kvserve_hpdps_b200.utils.logger import get_logger
from kvserve_hpdps_b200.utils.stats import timeline, write_compression_stats, write_decode_stats

try:  # vLLM is optional for importing this module (unit tests mock it)
    from vllm.distributed.kv_transfer.kv_connector.v1.base import (KVConnectorBase_V1,
                                                                   KVConnectorMetadata,
                                                                   KVConnectorRole)
except Exception:  # noqa: BLE001
    class KVConnectorMetadata:  # type: ignore[no-redef]
        pass

    class KVConnectorRole:  # type: ignore[no-redef]
        SCHEDULER = 0
        WORKER = 1

    class KVConnectorBase_V1:  # type: ignore[no-redef]
        def __init__(self, vllm_config, role, kv_cache_config=None):
            self._vllm_config = vllm_config
            self._role = role
            self._connector_metadata = None

        @property
        def role(self):
            return self._role

        def bind_connector_metadata(self, m):
            self._connector_metadata = m

        def clear_connector_metadata(self):
            self._connector_metadata = None

        def _get_connector_metadata(self):
            return self._connector_metadata

if TYPE_CHECKING:
    pass

from kvserve_hpdps_b200.utils.tracing import nvtx  # noqa: E402

logger = get_logger(__name__)

LOAD_TIMEOUT_S = float(os.environ.get("KVSERVE_LOAD_TIMEOUT_S", "60"))
CONTROLLER_FEEDBACK_TTL_S = 300.0  # as the adapter's controller contexts
STATS_ENTRY_TTL_S = 30.0  # unreported statistics entries of finished requests
# a received message no scheduled request claims within this time is released
UNCLAIMED_TTL_S = float(os.environ.get("KVSERVE_UNCLAIMED_TTL_S", "600"))


def normalize_overlap_mode(mode) -> str:
    """``off`` or ``stream``.  The reference's ``tq`` and ``full`` modes
    (per-layer transform/quantize on a side stream, codec and send at step
    end) map to ``off``: its step-end chain already runs every layer of a
    request in one launch per stage.  Anything else is ``off`` with a
    warning."""
    m = str(mode or "off").lower()
    if m in ("off", "stream"):
        return m
    if m in ("tq", "full"):
        logger.info("overlap mode %r: the fused step-end chain covers it; using 'off'", m)
        return "off"
    logger.warning("unknown overlap mode %r; using 'off'", mode)
    return "off"
DEFAULT_MAX_CHUNK_BYTES = 512 * 1024 * 1024
_LAYER_RE = re.compile(r"layers?\.(\d+)")


def layer_index(name: str) -> int:
    """Physical layer index parsed from a vLLM layer name
    ('model.layers.10.self_attn.attn' -> 10)."""
    m = _LAYER_RE.search(name)
    return int(m.group(1)) if m else 0


def _blocks_outer(kv_layer: torch.Tensor) -> bool:
    """True for a ``[num_blocks, 2, ...]`` (FlashInfer) layer, False for
    ``[2, num_blocks, ...]`` (FlashAttention); the block utilities tell the
    two apart the same way."""
    return kv_layer.shape[0] != 2 and kv_layer.dim() > 1 and kv_layer.shape[1] == 2


def max_chunk_bytes() -> int:
    raw = os.environ.get("KVSERVE_MAX_NCCL_CHUNK_BYTES")
    try:
        v = int(raw) if raw else DEFAULT_MAX_CHUNK_BYTES
    except ValueError:
        v = DEFAULT_MAX_CHUNK_BYTES
    return v if v > 0 else DEFAULT_MAX_CHUNK_BYTES


@dataclass
class ReqMeta:
    request_id: str
    transfer_id: str
    token_ids: list[int]
    block_ids: list[int]
    slot_mapping: torch.Tensor


@dataclass
class CompressedKVConnectorMetadata(KVConnectorMetadata):
    requests: list[ReqMeta] = field(default_factory=list)

    def add_request(self, request_id: str, transfer_id: str, token_ids: list[int],
                    block_ids: list[int], block_size: int) -> None:
        self.requests.append(ReqMeta(request_id, transfer_id, list(token_ids), list(block_ids),
                                     make_slot_mapping(token_ids, block_ids, block_size)))


class CompressedKVConnector(KVConnectorBase_V1):
    def __init__(self, vllm_config, role, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        cfg = vllm_config.kv_transfer_config
        self.is_producer = bool(cfg.is_kv_producer)
        self._block_size = int(vllm_config.cache_config.block_size)
        extra = dict(getattr(cfg, "kv_connector_extra_config", None) or {})
        self._compression_cfg = extra.get("compression")
        self._transport_kind = os.environ.get("KVSERVE_TRANSPORT", extra.get("transport", "auto"))
        # scheduler state
        self._requests_need_load: dict[str, tuple[Any, list[int]]] = {}
        self._request_transfer_ids: dict[str, str] = {}
        self.chunked_prefill: dict[str, tuple[list[int], list[int]]] = {}
        # model shapes
        mc, pc = vllm_config.model_config, vllm_config.parallel_config
        self._num_kv_heads = int(mc.get_num_kv_heads(pc))
        self._head_size = int(mc.get_head_size())
        try:
            self._num_layers = int(mc.get_num_layers(pc))
        except Exception:  # noqa: BLE001
            self._num_layers = int(getattr(mc.hf_text_config, "num_hidden_layers", 0))
        self._model_name = os.path.basename(str(mc.model).rstrip("/"))
        self._tp_rank, self._tp_size = 0, 1
        # overlap mode
        self._overlap_mode = str(extra.get("overlap", "off"))
        if isinstance(self._compression_cfg, dict) and "overlap" in self._compression_cfg:
            self._overlap_mode = self._compression_cfg.get("overlap", "off")
        self._overlap_mode = os.environ.get("KVSERVE_OVERLAP_MODE", self._overlap_mode)
        self._overlap_mode = normalize_overlap_mode(self._overlap_mode)
        prio = int(self._compression_cfg.get("side_stream_priority", 0)) \
            if isinstance(self._compression_cfg, dict) else 0
        self._side_priority = int(os.environ.get("KVSERVE_SIDE_PRIORITY", prio))
        self._async_send = os.environ.get("KVSERVE_ASYNC_SEND", "0") == "1" and self.is_producer
        # worker state
        self._compressor = None
        self._transport = None
        self._kv_caches: dict[str, torch.Tensor] = {}
        self._layer_refs: dict[str, torch.Tensor] = {}
        self._save_times: dict[str, list[float]] = defaultdict(list)
        self._worker_received: dict[str, deque] = defaultdict(deque)
        self._partial: dict[int, dict] = {}  # records with members still to decode
        self._step_reqs: dict[str, ReqMeta] = {}
        self._got: dict[str, int] = {}
        self._pending_layers: dict[str, set] = {}
        self._layer_events: dict[str, Any] = {}
        self._layer_wise = False
        self._load_stream = None
        self._fc = None
        self._deadline = 0.0
        self._side_stream = None
        self._streamed = False  # this step's layers were sent from save_kv_layer
        self._expected_msgs: dict[str, int] = {}
        self._rid2tid: dict[str, str] = {}
        self._pending_send_rids: set[str] = set()
        self._err_monitor = None
        # consumer: blocks whose load failed this step, handed to vLLM's
        # kv_load_failure_policy by get_block_ids_with_load_errors()
        self._load_errors: set[int] = set()
        # consumer: transfer ids whose load failed -> when; their messages
        # that arrive late are released instead of queued for good
        self._abandoned: dict[str, float] = {}
        # interval statistics for vLLM's connector-stats logging / Prometheus;
        # message key -> (original bytes, compress ms) of compressed messages
        # not yet reported sent by the transport
        self._xfer_stats = KVServeConnectorStats()
        self._sent_orig: dict[str, deque] = defaultdict(deque)
        self._sent_lock = threading.Lock()
        self._sent_retired: deque = deque()  # (time, transfer ids) whose messages are out
        # controller feedback: transfer id -> (request id, compress ms, time) until the
        # transport reports the message sent; completions queued by its thread
        self._ctl_wait: dict[str, tuple[str, float, float]] = {}
        self._ctl_done: deque = deque()
        # transfer id -> (request id, original bytes, reserved wire bytes, compress ms,
        # prefill span ms): compression statistics written once the message is out
        self._stats_wait: dict[str, tuple] = {}
        self._listening = False
        if role == KVConnectorRole.WORKER:
            self._init_worker(cfg)

    # ================================================================ worker init
    def _init_worker(self, cfg) -> None:
        try:
            from vllm.distributed.parallel_state import (get_tensor_model_parallel_rank,
                                                         get_tensor_model_parallel_world_size,
                                                         get_world_group)
            local_rank = get_world_group().local_rank
            self._tp_rank = get_tensor_model_parallel_rank()
            self._tp_size = get_tensor_model_parallel_world_size()
        except Exception:  # noqa: BLE001
            local_rank = torch.cuda.current_device() if torch.cuda.is_available() else 0
        self._local_rank = local_rank
        self._transport = self._build_transport(cfg, local_rank, self._tp_rank)
        self._watch_transport()
        if self._compression_cfg is not None:
            comp = self._get_compressor()
            if comp is not None:
                comp.warmup(self._block_size)
        if self.is_producer and self._overlap_mode == "stream" and torch.cuda.is_available():
            self._side_stream = torch.cuda.Stream(priority=self._side_priority)
        logger.info("worker init: producer=%s tp=%d/%d transport=%s compression=%s overlap=%s",
                    self.is_producer, self._tp_rank, self._tp_size,
                    type(self._transport).__name__, self._compression_cfg is not None,
                    self._overlap_mode)

    def _build_transport(self, cfg, local_rank: int, channel_rank: int):
        kind = self._transport_kind
        if kind == "fake":
            return None  # tests attach a transport explicitly
        if kind == "auto":
            kind = "p2p" if torch.cuda.is_available() and torch.cuda.device_count() > 1 else "nccl"
        if kind == "p2p":
            from kvserve_hpdps_b200.parallel.p2p_transport import P2PTransport
            ring = int(os.environ.get("KVSERVE_RING_BYTES", str(2 << 30)))
            return P2PTransport(self.is_producer, cfg.kv_ip, cfg.kv_port, local_rank,
                                channel_rank, ring_bytes=ring)
        from kvserve_hpdps_b200.parallel.nccl_transport import NcclTransport
        return NcclTransport(self.is_producer, cfg.kv_ip, cfg.kv_port, local_rank, channel_rank)

    def attach_transport(self, transport) -> None:
        self._transport = transport
        self._listening = False
        self._watch_transport()

    # ----------------------------------------------- controller feedback
    def _watch_transport(self) -> None:
        """Producer: hear from the transport when a message has left, so the
        controller learns from compress + transfer time (the reference feeds
        it the host time of compress + enqueue, taken before the transfer)."""
        tr = self._transport
        if self.is_producer and not self._listening and hasattr(tr, "add_sent_listener"):
            tr.add_sent_listener(self._on_sent)
            self._listening = True

    def _on_sent(self, request_id: str, transfer_ids: list[str], latency_ms: float,
                 nbytes: Optional[int] = None) -> None:
        # transport thread: only queue controller updates (the engine thread
        # applies them); compression statistics wait for the exact size on
        # the wire (a coded stream's length is known only on the device)
        with self._sent_lock:
            q = self._sent_orig.get(request_id)
            orig, cms = q.popleft() if q else (None, 0.0)
            if q is not None and not q:
                self._sent_orig.pop(request_id, None)
        if nbytes:
            self._xfer_stats.record_sent(orig if orig else nbytes, nbytes, cms, latency_ms)
        for t in transfer_ids:
            if t in self._ctl_wait:
                self._ctl_done.append((t, latency_ms))
            stat = self._stats_wait.pop(t, None)
            if stat is not None:
                rid, orig, wire, ms, span = stat
                write_compression_stats(rid, t, orig, nbytes if nbytes else wire,
                                        compress_ms=ms, prefill_span_ms=span)

    def _kv_bytes(self, num_layers: int, tokens: int, cache: torch.Tensor) -> int:
        """Bytes of ``tokens`` tokens of K and V over ``num_layers`` layers."""
        return (num_layers * 2 * tokens * self._num_kv_heads * self._head_size
                * cache.element_size())

    def _expect_sent(self, key: str, original_bytes: Optional[int] = None) -> Optional[list]:
        """Before a message goes to the transport under ``key``: queue its
        statistics entry ``[original bytes (None: raw KV), compress ms]``,
        completed when the transport reports the message sent (exact wire
        bytes, transfer time; a transport reports the messages of one key in
        send order).  Returns the entry, or None without a listener."""
        if not self._listening:
            return None
        entry = [original_bytes, 0.0]
        with self._sent_lock:
            self._sent_orig[key].append(entry)
        return entry

    def _settle_sent(self, key: str, entry: Optional[list], sent: bool,
                     original_bytes: Optional[int] = None, wire_bytes: int = 0,
                     compress_ms: float = 0.0) -> None:
        """After the send call: a message that did not go out takes its entry
        back; without a listener a sent compressed message is recorded now."""
        if entry is not None:
            entry[1] = compress_ms
            if not sent:
                with self._sent_lock:
                    q = self._sent_orig.get(key)
                    if q and q[-1] is entry:
                        q.pop()
                    if q is not None and not q:
                        self._sent_orig.pop(key, None)
        elif sent and original_bytes:
            self._xfer_stats.record_sent(original_bytes, wire_bytes, compress_ms, 0.0)

    def _apply_controller_feedback(self) -> None:
        comp = self._compressor
        while self._ctl_done:
            tid, latency_ms = self._ctl_done.popleft()
            entry = self._ctl_wait.pop(tid, None)
            if entry is not None and comp is not None:
                comp.update_controller(entry[0], entry[1] + latency_ms)
        if self._ctl_wait:  # messages that never left (refused, dropped)
            cutoff = time.monotonic() - CONTROLLER_FEEDBACK_TTL_S
            for tid in [t for t, e in self._ctl_wait.items() if e[2] < cutoff]:
                self._ctl_wait.pop(tid, None)

    def _get_compressor(self):
        if self._compression_cfg is None:
            return None
        if self._compressor is None:
            from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter
            bw = getattr(self._transport, "bandwidth_mbps", None) if self.is_producer else None
            self._compressor = KVCompressionAdapter(
                self._compression_cfg, self._num_kv_heads, self._head_size,
                model_name=self._model_name, tp_rank=self._tp_rank, tp_size=self._tp_size,
                num_layers=self._num_layers or None,
                bandwidth_fn=bw)  # controller mode: device-timed link bandwidth
        return self._compressor

    @classmethod
    def get_required_kvcache_layout(cls, vllm_config) -> Optional[str]:
        mc = getattr(vllm_config, "model_config", None)
        if mc is None or getattr(mc, "use_mla", False):
            return None
        return "NHD"

    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]) -> None:
        self._kv_caches = dict(kv_caches)

    # ================================================================ producer
    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata: Any,
                      **kwargs: Any) -> None:
        if not self.is_producer:
            return
        meta = self._get_connector_metadata()
        if not isinstance(meta, CompressedKVConnectorMetadata) or not meta.requests:
            return
        self._layer_refs[layer_name] = kv_layer
        now = time.monotonic()
        for rm in meta.requests:
            self._save_times[rm.request_id].append(now)
        comp = self._get_compressor()
        if self._side_stream is not None and comp is None and kv_layer.is_cuda:
            # raw KV, layer by layer: each request's blocks of this layer go
            # out as their own message on the side stream (the consumer counts
            # one message per layer for each transfer id)
            ready = torch.cuda.current_stream().record_event()
            with torch.cuda.stream(self._side_stream):
                self._side_stream.wait_event(ready)
                for rm in meta.requests:
                    self._expect_sent(rm.transfer_id)
                    if hasattr(self._transport, "send_paged"):
                        self._transport.send_paged(rm.transfer_id, [layer_name], [kv_layer],
                                                   rm.block_ids)
                    else:
                        raw = extract_kv_from_layer_by_blocks(kv_layer, rm.block_ids).unsqueeze(0)
                        self._transport.send(rm.transfer_id, [layer_name], raw)
                    self._expected_msgs[rm.transfer_id] = self._num_layers
            self._streamed = True
            return
        if self._side_stream is not None and comp is not None and comp.supports_paged():
            self._streamed = True
            ready = torch.cuda.current_stream().record_event()
            requests = [(rm.block_ids, len(rm.token_ids)) for rm in meta.requests]
            tids = [rm.transfer_id for rm in meta.requests]
            try:
                with torch.cuda.stream(self._side_stream):
                    self._side_stream.wait_event(ready)
                    # one grouped message for the layer; on the NVLink ring the
                    # producer kernels store it straight into the consumer's memory
                    t0 = time.monotonic()
                    orig = sum(self._kv_bytes(1, n, kv_layer) for _, n in requests)
                    entry, info = self._expect_sent(tids[0], orig), None
                    try:
                        info = comp.send_paged_requests(self._transport, tids[0],
                                                        add_sentinel([layer_name]), [kv_layer],
                                                        [layer_index(layer_name)], requests,
                                                        member_tids=tids)
                    finally:
                        self._settle_sent(tids[0], entry, bool(info and info["wire_nbytes"]),
                                          orig, info["wire_nbytes"] if info else 0,
                                          (time.monotonic() - t0) * 1e3)
            except Exception:  # noqa: BLE001
                # as in the off mode: a compression failure sends this layer's raw
                # KV, one message per request (the consumer still counts one
                # message per layer for each transfer id)
                logger.exception("compression of %s failed; sending raw KV", layer_name)
                info = None
            if info is None:  # failed, or the controller picked no compression
                with torch.cuda.stream(self._side_stream):
                    for rm in meta.requests:
                        raw = extract_kv_from_layer_by_blocks(kv_layer, rm.block_ids).unsqueeze(0)
                        self._expect_sent(rm.transfer_id)
                        self._transport.send(rm.transfer_id, [layer_name], raw)
            for t in tids:
                self._expected_msgs[t] = self._num_layers

    def _send_compressed(self, tid: str, layer_names: list[str], cd, member_tids=None) -> int:
        wire = build_wire(cd, max_chunk_bytes())
        self._transport.send_bundle(tid, add_sentinel(layer_names), wire.meta, wire.body_chunks,
                                    wire.aux_tensors, member_tids=member_tids)
        return wire.nbytes

    def wait_for_save(self) -> None:
        if not self.is_producer:
            return
        meta = self._get_connector_metadata()
        if not isinstance(meta, CompressedKVConnectorMetadata):
            return
        timeline("P save_enter")
        self._apply_controller_feedback()
        if self._side_stream is not None:
            torch.cuda.current_stream().wait_stream(self._side_stream)
        if self._streamed:  # every layer already went out from save_kv_layer
            self._streamed = False
            self._finish_step(meta)
            timeline("P save_exit")
            return
        names = sorted(self._layer_refs, key=layer_index)
        comp = self._get_compressor()
        for rm in meta.requests:
            if not names:
                break
            rid, tid = rm.request_id, rm.transfer_id
            t0 = time.monotonic()
            span = self._prefill_span(rid)
            layers = [self._layer_refs[n] for n in names]
            use = comp  # this request's compressor (None: raw KV)
            if use is not None and use.supports_paged() and layers[0].is_cuda:
                orig = self._kv_bytes(len(layers), len(rm.token_ids), layers[0])
                entry, info = self._expect_sent(tid, orig), None
                try:
                    with nvtx("kvs.compress_send"):
                        info = use.send_paged_requests(
                            self._transport, tid, add_sentinel(names), layers,
                            [layer_index(n) for n in names], [(rm.block_ids, len(rm.token_ids))],
                            member_tids=[tid])
                except Exception:  # noqa: BLE001
                    # as the reference does: a compression failure sends the raw KV
                    logger.exception("compression of %s failed; sending raw KV", rid)
                    info = None
                self._settle_sent(tid, entry, bool(info and info["wire_nbytes"]), orig,
                                  info["wire_nbytes"] if info else 0,
                                  (time.monotonic() - t0) * 1e3)
                if info is not None:
                    self._expected_msgs[tid] = 1
                    compress_ms = (time.monotonic() - t0) * 1e3
                    stat = (rid, info["original_size"], info["wire_nbytes"], compress_ms, span)
                    ctl = getattr(use, "controller_mode", False)
                    if self._listening:  # written with the exact size once it is out
                        self._stats_wait[tid] = stat
                        if ctl:  # the paged path keys the controller context by transfer id
                            self._ctl_wait[tid] = (tid, compress_ms, time.monotonic())
                    else:
                        write_compression_stats(rid, tid, stat[1], stat[2], compress_ms=stat[3],
                                                prefill_span_ms=stat[4])
                        if ctl:
                            use.update_controller(tid, compress_ms)
                    continue
                use = None  # failed, or the controller picked no compression
            if use is None and hasattr(self._transport, "send_paged") and layers[0].is_cuda:
                # raw KV: one gather launch from the paged caches into the peer ring
                with nvtx("kvs.send_raw"):
                    self._expect_sent(tid)
                    self._transport.send_paged(tid, names, layers, rm.block_ids)
                self._expected_msgs[tid] = 1
                continue
            stacked = torch.stack([extract_kv_from_layer_by_blocks(l, rm.block_ids)
                                   for l in layers], 0)
            if use is not None and _blocks_outer(layers[0]):
                # compressors take [L, 2 (K, V), blocks, ...]; the raw path keeps
                # the caches' own order, which the consumer's caches share
                stacked = stacked.transpose(1, 2).contiguous()
            cd = use.compress(stacked, rid) if use is not None else None
            if cd is not None:
                compress_ms = (time.monotonic() - t0) * 1e3
                if self._listening:  # completed by _apply_controller_feedback
                    self._ctl_wait[tid] = (rid, compress_ms, time.monotonic())
                orig = stacked.numel() * stacked.element_size()
                entry = self._expect_sent(tid, orig)
                nbytes = self._send_compressed(tid, names, cd)
                self._settle_sent(tid, entry, True, orig, nbytes, (time.monotonic() - t0) * 1e3)
                if not self._listening:
                    use.update_controller(rid, (time.monotonic() - t0) * 1e3)
                write_compression_stats(rid, tid, stacked.numel() * stacked.element_size(), nbytes,
                                        compress_ms=(time.monotonic() - t0) * 1e3,
                                        prefill_span_ms=span)
            else:
                self._expect_sent(tid)
                self._transport.send(tid, names, stacked)
            self._expected_msgs[tid] = 1
        self._finish_step(meta)
        timeline("P save_exit")

    def _prefill_span(self, rid: str) -> float:
        ts = self._save_times.pop(rid, [])
        return (max(ts) - min(ts)) * 1e3 if len(ts) >= 2 else 0.0

    def _finish_step(self, meta) -> None:
        for rm in meta.requests:
            self._save_times.pop(rm.request_id, None)
            self._rid2tid[rm.request_id] = rm.transfer_id
        self._layer_refs.clear()
        if not self._async_send and self._transport is not None:
            self._transport.wait_for_sent()
            self._retire_sent_entries([rm.transfer_id for rm in meta.requests])

    def _retire_sent_entries(self, tids) -> None:
        """The requests' messages are out (or refused, or dropped): statistics
        entries still queued under their transfer ids belong to messages the
        transport never reported, and are dropped once the transport thread
        has had ample time for any late report (it may report a message just
        after the wait for it returned)."""
        now = time.monotonic()
        self._sent_retired.append((now, list(tids)))
        with self._sent_lock:
            while self._sent_retired and now - self._sent_retired[0][0] > STATS_ENTRY_TTL_S:
                for t in self._sent_retired.popleft()[1]:
                    self._sent_orig.pop(t, None)
                    self._stats_wait.pop(t, None)  # JSONL rows of messages never reported

    def get_finished(self, finished_req_ids: set[str]):
        if self.is_producer:
            self._apply_controller_feedback()
        if not self._async_send:
            return None, None
        self._pending_send_rids |= set(finished_req_ids or ())
        done = set()
        failed = getattr(self._transport, "failed_layers", None)
        for rid in list(self._pending_send_rids):
            tid = self._rid2tid.get(rid)
            # refused or unsent messages count as out: the blocks are free to reuse
            out = 0 if tid is None else self._transport.sent_layers(tid) + (
                failed(tid) if failed is not None else 0)
            if tid is None or out >= self._expected_msgs.get(tid, 1):
                done.add(rid)
                n_failed = failed(tid) if (failed is not None and tid is not None) else 0
                if n_failed:
                    self._xfer_stats.record_failed_send(n_failed)
        self._pending_send_rids -= done
        for rid in done:
            tid = self._rid2tid.pop(rid, None)
            if tid is not None:
                self._retire_sent_entries([tid])
                self._transport.clear_sent(tid)
                self._expected_msgs.pop(tid, None)
        return (done or None), None

    # ================================================================ consumer
    # Received messages become records shared by every member request they
    # carry (a stream-mode message holds one layer of every request of the
    # producer's step): {"names", "payload", "members", "decoded", "prepared",
    # "cd"}.  A record is queued under each member's transfer id; decoding it
    # for the members scheduled now marks them decoded, and its ring space goes
    # back once every member has been decoded.
    def start_load_kv(self, forward_context: Any, **kwargs: Any) -> None:
        if self.is_producer:
            return
        timeline("D load_enter")
        meta = self._get_connector_metadata()
        if isinstance(meta, CompressedKVConnectorMetadata):
            for rm in meta.requests:  # scheduled to load (again): wanted after all
                self._abandoned.pop(rm.transfer_id, None)
        self._drain()
        if not isinstance(meta, CompressedKVConnectorMetadata):
            return
        self._fc = forward_context
        self._step_reqs = {rm.transfer_id: rm for rm in meta.requests}
        self._drop_abandoned()
        self._got = {t: 0 for t in self._step_reqs}
        # one deadline for the step: with a dead producer the step returns
        # after LOAD_TIMEOUT_S, not after that long for each of its requests
        self._deadline = time.monotonic() + LOAD_TIMEOUT_S
        names = sorted(self._kv_caches, key=layer_index)
        self._layer_wise = (self._overlap_mode == "stream" and bool(names)
                            and len(names) == self._num_layers and torch.cuda.is_available()
                            and bool(meta.requests))
        if self._layer_wise:
            # Layer-wise load: decode what has arrived on the load stream and
            # return; wait_for_layer_load(l) waits (host: for layer l's header,
            # device: for its decode) only for layer l, so the forward of the
            # first layers runs while later layers are still on the wire.
            if self._load_stream is None:
                self._load_stream = torch.cuda.Stream()
            # decodes start after every earlier kernel of the forward stream
            # (blocks just handed to these requests may have been read by it)
            self._load_stream.wait_stream(torch.cuda.current_stream())
            self._layer_events = {}
            self._pending_layers = {t: set(names) for t in self._step_reqs}
            self._decode_available()
        else:
            self._pending_layers = {}
            streaming = self._overlap_mode == "stream" and self._num_layers > 0
            need = self._num_layers if streaming else 1
            while True:
                self._decode_available()
                if all(self._got[t] >= need for t in self._step_reqs):
                    break
                if time.monotonic() > self._deadline:
                    late = [t for t in self._step_reqs if self._got[t] < need]
                    for t in late:
                        logger.warning("timeout loading KV of %s (transfer %s): %d/%d "
                                       "messages", self._step_reqs[t].request_id, t,
                                       self._got[t], need)
                    self._fail_load(late)
                    break
                self._wait_header()
                self._drain()
        self._poll_device_errors(bool(meta.requests))
        timeline("D load_exit")

    def _wait_header(self) -> None:
        waiter = getattr(self._transport, "wait_received", None)
        if waiter is not None:
            waiter(0.002)  # wakes as soon as a message header arrives
        else:
            time.sleep(0.002)

    def _poll_device_errors(self, any_requests: bool) -> None:
        """Device-side failures of earlier loads (flag timeouts, checksum
        mismatches, corrupt streams), read without waiting on the GPU."""
        if not (torch.cuda.is_available() and any_requests):
            return
        from kvserve_hpdps_b200.ops import kernels as K
        if self._err_monitor is None:
            self._err_monitor = K.ErrorMonitor(torch.device("cuda", torch.cuda.current_device()))
        code = self._err_monitor.poll()
        if code:
            logger.error("device error %d (%s) while loading KV in an earlier step", code,
                         K.ERR_NAMES.get(code, "?"))

    def wait_for_layer_load(self, layer_name: str) -> None:
        """Stream mode: before layer ``layer_name`` runs, make sure its KV of
        every request of the step is decoded -- the host waits (bounded by
        the step's deadline) only until that layer's message headers have
        arrived, and the forward stream waits on the device for that layer's
        decode, not for the whole request."""
        if self.is_producer or not self._layer_wise:
            return
        pend = self._pending_layers
        while any(layer_name in p for p in pend.values()):
            self._drain()
            self._decode_available()
            if not any(layer_name in p for p in pend.values()):
                break
            if time.monotonic() > self._deadline:
                late = [t for t, p in pend.items() if layer_name in p]
                logger.warning("timeout loading layer %s of %d request(s) (%s)", layer_name,
                               len(late), ", ".join(late[:4]))
                for t in late:
                    pend[t].discard(layer_name)
                self._fail_load(late)
                break
            self._wait_header()
        ev = self._layer_events.get(layer_name)
        if ev is not None:
            torch.cuda.current_stream().wait_event(ev)

    @staticmethod
    def _members(tid: str, payload: Any) -> list[str]:
        """Transfer ids a received message carries (grouped messages name
        their members in the wire metadata)."""
        if isinstance(payload, dict) and payload.get("__bundle__"):
            inner = (payload.get("meta") or {}).get("metadata")
            if isinstance(inner, dict) and inner.get("member_tids"):
                return [str(t) for t in inner["member_tids"]]
        return [tid]

    def _drain(self) -> None:
        for tid, msgs in (self._transport.drain_received() or {}).items():
            for names, payload in msgs:
                members = self._members(tid, payload)
                # members whose load already failed will not be scheduled to
                # load again (vLLM recomputes or fails them): count them done
                gone = {t for t in members if t in self._abandoned}
                rec = {"names": names, "payload": payload, "members": set(members),
                       "decoded": set(gone), "prepared": False, "cd": None,
                       "arrived": time.monotonic()}
                if gone and gone == rec["members"]:
                    self._release_late(rec)
                    continue
                for t in members:
                    if t not in gone:
                        self._worker_received[t].append(rec)

    def _release_late(self, rec: dict) -> None:
        """A message nobody will decode (its requests' loads failed before
        it arrived): its ring space goes back at once."""
        logger.info("releasing a late message for %s", ", ".join(sorted(rec["members"])))
        self._release_rec(rec)

    def _drop_abandoned(self) -> None:
        """Queued messages of requests whose load failed in an earlier step,
        and messages no scheduled request has claimed for ``UNCLAIMED_TTL_S``
        (a request the decode engine never got), are dropped (released once
        no other member needs them); failed transfer ids are forgotten after
        ten load timeouts."""
        stale = time.monotonic() - UNCLAIMED_TTL_S
        for t in [t for t, q in self._worker_received.items()
                  if t not in self._step_reqs and q and q[0].get("arrived", stale) < stale]:
            logger.warning("no request claimed the KV of transfer %s for %.0f s; dropping it",
                           t, UNCLAIMED_TTL_S)
            self._abandoned.setdefault(t, time.monotonic())
        if not self._abandoned:
            return
        for t in [t for t in self._worker_received if t in self._abandoned]:
            for rec in self._worker_received.pop(t):
                rec["decoded"].add(t)
                if rec["decoded"] >= rec["members"]:
                    self._release_late(rec)
        cutoff = time.monotonic() - 10 * LOAD_TIMEOUT_S
        for t in [t for t, when in self._abandoned.items() if when < cutoff]:
            self._abandoned.pop(t, None)

    def _layer_cache(self, name: str, forward_context: Any) -> Optional[torch.Tensor]:
        t = self._kv_caches.get(name)
        if t is not None:
            return t
        if forward_context is None:
            return None
        layer = getattr(forward_context, "no_compile_layers", {}).get(name)
        cache = getattr(layer, "kv_cache", None) if layer is not None else None
        if cache is None:
            return None
        return cache[getattr(forward_context, "virtual_engine", 0)]

    def _decode_available(self) -> None:
        """Decode every queued record of the step's requests, for the members
        scheduled now.  Layer-wise mode puts the kernels on the load stream
        and records one event per decoded layer."""
        ctx = torch.cuda.stream(self._load_stream) if self._layer_wise else nullcontext()
        with ctx:
            for tid in list(self._step_reqs):
                q = self._worker_received.get(tid)
                while q:
                    rec = q.popleft()
                    if tid not in rec["decoded"]:
                        self._decode_record(rec)
                if q is not None and not q:
                    self._worker_received.pop(tid, None)
        self._sweep_partial()

    def _decode_record(self, rec: dict) -> None:
        now = [t for t in rec["members"] if t in self._step_reqs and t not in rec["decoded"]]
        if not now:
            return
        names, payload = rec["names"], rec["payload"]
        plain = strip_sentinel(names) if is_compressed_layer_names(names) else list(names)
        if payload is None:
            logger.error("transport reported a failed transfer for %s", ", ".join(now))
            self._fail_load(now)
            self._mark(rec, now, plain)
            return
        tr = self._transport
        dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() \
            else torch.device("cpu")
        t0 = time.monotonic()
        try:
            if not rec["prepared"] and hasattr(tr, "prepare"):
                tr.prepare(payload, dev)  # bounded device flag wait + checksum, once
            rec["prepared"] = True
            with nvtx("kvs.inject"):
                self._inject_record(rec, now, plain, payload)
            ms = (time.monotonic() - t0) * 1e3
            for t in now:
                self._xfer_stats.record_decode(ms)
                if is_compressed_layer_names(names):
                    write_decode_stats(self._step_reqs[t].request_id, t, ms)
        except Exception as e:  # noqa: BLE001
            logger.error("decode of %s failed: %s", ", ".join(now), e)
            self._fail_load(now)
        finally:
            self._mark(rec, now, plain)
            if rec["decoded"] >= rec["members"]:
                self._release_rec(rec, dev)  # after the decode queued on this stream
            else:
                rec.setdefault("t", time.monotonic())
                self._partial[id(rec)] = rec

    def _fail_load(self, tids) -> None:
        """The KV of these requests of the step did not (fully) arrive: their
        blocks are reported to vLLM, which recomputes them or fails the
        request (``kv_load_failure_policy``), instead of decoding with stale
        blocks."""
        now = time.monotonic()
        for t in tids:
            rm = self._step_reqs.get(t)
            if rm is not None:
                self._load_errors.update(int(b) for b in rm.block_ids)
                self._xfer_stats.record_failed_load()
                self._abandoned[t] = now

    def get_kv_connector_stats(self) -> Optional[KVServeConnectorStats]:
        """This worker's transfer statistics since the last call (None when
        there are none); vLLM aggregates them over workers and logs them."""
        if self._xfer_stats.is_empty():
            return None
        return self._xfer_stats.clone_and_reset()

    @classmethod
    def build_kv_connector_stats(cls, data: Optional[dict] = None) -> KVServeConnectorStats:
        return KVServeConnectorStats(data={k: list(v) for k, v in (data or {}).items()})

    @classmethod
    def build_prom_metrics(cls, vllm_config, metric_types, labelnames, per_engine_labelvalues):
        return KVServePromMetrics(vllm_config, metric_types, labelnames, per_engine_labelvalues)

    def get_block_ids_with_load_errors(self) -> set[int]:
        """Blocks of the requests whose load failed in this step (a failed
        payload, a decode error, or the step's load timeout).  Failures the
        device reports later (a flag timeout or checksum mismatch inside a
        kernel, seen by the error monitor) are logged only: the forward has
        already run by then.  The reference decodes with whatever the blocks
        hold in every case (kvserve_v1/connector/compressed_kv_connector.py:
        423-441)."""
        out, self._load_errors = self._load_errors, set()
        return out

    def _mark(self, rec: dict, members: list[str], names: list[str]) -> None:
        rec["decoded"].update(members)
        for t in members:
            if t in self._got:
                self._got[t] += 1
            pend = self._pending_layers.get(t)
            if pend:
                pend.difference_update(names)
        if self._layer_wise:
            ev = self._load_stream.record_event()
            for n in names:
                self._layer_events[n] = ev

    def _sweep_partial(self) -> None:
        """Grouped records some of whose members were never scheduled here
        give their ring space back after twice the load timeout.  The members
        still waiting lose the record with it: a later load of theirs fails
        cleanly (reported to vLLM) instead of decoding memory the producer may
        have reused."""
        if not self._partial:
            return
        cutoff = time.monotonic() - 2 * LOAD_TIMEOUT_S
        now = time.monotonic()
        for key, rec in list(self._partial.items()):
            if rec.get("t", 0.0) < cutoff:
                for t in rec["members"] - rec["decoded"]:
                    q = self._worker_received.get(t)
                    if q is not None:  # by identity: records hold tensors
                        rest = deque(r for r in q if r is not rec)
                        if rest:
                            self._worker_received[t] = rest
                        else:
                            self._worker_received.pop(t, None)
                    self._abandoned.setdefault(t, now)
                self._release_rec(rec)

    def _release_rec(self, rec: dict, device=None) -> None:
        """Return a record's ring space, once, whichever path gets there first."""
        self._partial.pop(id(rec), None)
        if rec.get("released"):
            return
        rec["released"] = True
        if hasattr(self._transport, "release"):
            if device is None:
                self._transport.release(rec["payload"])
            else:
                self._transport.release(rec["payload"], device)

    def _inject_record(self, rec: dict, members: list[str], names: list[str],
                       payload: Any) -> None:
        fc = self._fc
        if is_compressed_layer_names(rec["names"]):
            if rec["cd"] is None:
                rec["cd"] = restore_from_wire(CompressedWire(payload["meta"], payload["body_chunks"],
                                                             payload["aux_tensors"]))
            cd = rec["cd"]
            md = cd.metadata or {}
            if md.get("num_heads") is not None:
                self._check_heads(int(md["num_heads"]))
            comp = self._get_compressor()
            if md.get("layout") in ("items", "items_packed"):
                caches = [self._layer_cache(n, fc) for n in names]
                if any(c is None for c in caches):
                    raise RuntimeError("missing KV cache tensor for a layer of the message")
                tids = md["member_tids"]
                if len(tids) == 1:
                    rm = self._step_reqs[members[0]]
                    comp.decompress_paged_requests(cd, caches,
                                                   [(rm.block_ids, md["member_tokens"][0])])
                else:  # one launch for every member scheduled now
                    sel = {i: self._step_reqs[t].block_ids for i, t in enumerate(tids)
                           if t in members}
                    comp.decompress_members(cd, caches, sel)
                return
            kv = comp.decompress(cd)
            if kv is None:
                raise RuntimeError("decompression returned None")
            self._check_heads(int(kv.shape[-2]))  # [L, 2, blocks, block_size, heads, dim]
            rm = self._step_reqs[members[0]]
            for i, name in enumerate(names):
                cache = self._layer_cache(name, fc)
                if cache is not None:  # kv[i] is [2 (K, V), blocks, ...]
                    part = kv[i].transpose(0, 1) if _blocks_outer(cache) else kv[i]
                    inject_kv_into_layer_by_blocks(cache, part, rm.block_ids, rm.request_id)
            return
        rm = self._step_reqs[members[0]]
        payload_t = payload["tensor"] if isinstance(payload, dict) and \
            payload.get("__ring_raw__") else payload
        caches = [self._layer_cache(n, fc) for n in names]
        if self._scatter_raw(rm, caches, payload, payload_t):
            return
        for cache, part in zip(caches, payload_t):
            if cache is not None:
                inject_kv_into_layer_by_blocks(cache, part, rm.block_ids, rm.request_id)

    def _check_heads(self, heads: int) -> None:
        if heads != self._num_kv_heads:
            raise ValueError(
                f"the message carries {heads} KV heads per rank but this consumer's caches hold "
                f"{self._num_kv_heads}: producer and consumer must run the same tensor-parallel "
                f"size (heterogeneous TP is not supported)")

    @staticmethod
    def _scatter_raw(rm: ReqMeta, caches: list, payload: Any, payload_t: Any) -> bool:
        """Scatter a raw ``[L, 2, nb, ...]`` device payload into every layer
        at this request's blocks in one launch.  Needs the same block count
        and block order on both sides; False leaves it to the per-layer
        path (which also handles partial overlaps)."""
        if not (isinstance(payload_t, torch.Tensor) and payload_t.is_cuda
                and payload_t.is_contiguous() and payload_t.dim() == 6):
            return False
        if any(c is None for c in caches) or payload_t.shape[0] != len(caches):
            return False
        if payload_t.shape[2] != len(rm.block_ids) or any(c.dtype != payload_t.dtype
                                                           for c in caches):
            return False
        from kvserve_hpdps_b200.ops import kernels as K
        order = payload.get("block_order", "nhd") if isinstance(payload, dict) else "nhd"
        try:
            orders = {K._raw_block_layout(c)[1] for c in caches}
        except ValueError:
            return False
        if orders != {order} or any(c.shape[2:] != payload_t.shape[3:] for c in caches):
            return False
        ids = [int(b) for b in rm.block_ids]
        raw = K.RawItems(caches, [(l, ids) for l in range(len(caches))])
        with nvtx("kvs.scatter_raw"):
            K.paged_raw(raw, payload_t.data_ptr(), gather=False)
        return True

    # ================================================================ scheduler
    def get_num_new_matched_tokens(self, request: Any, num_computed_tokens: int):
        if self.is_producer:
            return 0, False
        n = len(request.prompt_token_ids) - 1 - num_computed_tokens
        return (n, False) if n > 0 else (0, False)

    def update_state_after_alloc(self, request: Any, blocks: Any, num_external_tokens: int) -> None:
        self._resolve_transfer_id(request.request_id, request)
        if not self.is_producer and num_external_tokens > 0:
            self._requests_need_load[request.request_id] = (request, blocks.get_block_ids()[0])

    def build_connector_meta(self, scheduler_output: Any) -> CompressedKVConnectorMetadata:
        meta = CompressedKVConnectorMetadata()
        for nr in scheduler_output.scheduled_new_reqs:
            if self.is_producer:
                n = scheduler_output.num_scheduled_tokens[nr.req_id] + nr.num_computed_tokens
                prompt = nr.prompt_token_ids or []
                if n < len(prompt):
                    self.chunked_prefill[nr.req_id] = (list(nr.block_ids[0]), prompt)
                    continue
                meta.add_request(nr.req_id, self._resolve_transfer_id(nr.req_id), prompt,
                                 nr.block_ids[0], self._block_size)
            elif nr.req_id in self._requests_need_load:
                meta.add_request(nr.req_id, self._resolve_transfer_id(nr.req_id),
                                 nr.prompt_token_ids or [], nr.block_ids[0], self._block_size)
                self._requests_need_load.pop(nr.req_id)
        cached = scheduler_output.scheduled_cached_reqs
        resumed = getattr(cached, "resumed_req_ids", set()) or set()
        for i, rid in enumerate(cached.req_ids):
            computed = cached.num_computed_tokens[i]
            new_blocks = cached.new_block_ids[i]
            is_resumed = rid in resumed
            if self.is_producer:
                if rid not in self.chunked_prefill:
                    continue
                n = scheduler_output.num_scheduled_tokens[rid] + computed
                blocks = list(new_blocks[0]) if new_blocks is not None else []
                if not is_resumed:
                    blocks = self.chunked_prefill[rid][0] + blocks
                prompt = self.chunked_prefill[rid][1]
                if n < len(prompt):
                    self.chunked_prefill[rid] = (blocks, prompt)
                    continue
                meta.add_request(rid, self._resolve_transfer_id(rid), prompt, blocks,
                                 self._block_size)
                self.chunked_prefill.pop(rid, None)
                continue
            if not is_resumed:
                continue
            if rid in self._requests_need_load:
                req, _ = self._requests_need_load.pop(rid)
                tokens = list(req.all_token_ids[:computed + 1])
                blocks = list(new_blocks[0]) if new_blocks is not None else []
                meta.add_request(rid, self._resolve_transfer_id(rid, req), tokens, blocks,
                                 self._block_size)
        return meta

    def request_finished(self, request: Any, block_ids: list[int]):
        self.chunked_prefill.pop(request.request_id, None)
        self._request_transfer_ids.pop(request.request_id, None)
        if not self.is_producer:
            self._requests_need_load.pop(request.request_id, None)
            return False, None
        return (True, None) if self._async_send else (False, None)

    def _resolve_transfer_id(self, request_id: str, request: Any = None) -> str:
        if request is not None:
            params = getattr(request, "kv_transfer_params", None)
            if params and params.get("transfer_id"):
                self._request_transfer_ids[request_id] = str(params["transfer_id"])
            elif request_id not in self._request_transfer_ids:
                logger.warning("request %s has no transfer_id; using the request id", request_id)
        return self._request_transfer_ids.get(request_id, request_id)

    def shutdown(self) -> None:
        comp = self._compressor
        if comp is not None and hasattr(comp, "save_controller_state"):
            comp.save_controller_state()
        if self._transport is not None and hasattr(self._transport, "close"):
            self._transport.close()
