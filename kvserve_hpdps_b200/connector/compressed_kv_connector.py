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
* consumer: ``start_load_kv`` drains the transport, waits (bounded) for each
  scheduled request's payloads and decodes them straight into the registered
  paged caches at the consumer's block ids (fused dequantize + inverse
  transform + scatter); raw payloads are scattered with the block-copy kernel.

Transports: ``"p2p"`` (NVLink receive ring, producer kernels store into the
consumer's memory), ``"nccl"`` (reference protocol over a torch NCCL group)
or ``"auto"`` (p2p when both GPUs are visible to the producer, else nccl);
``kv_connector_extra_config["transport"]`` or ``KVSERVE_TRANSPORT`` selects.
"""

from __future__ import annotations

import os
import re
import time
from collections import defaultdict, deque
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any, Optional

import torch

from kvserve_hpdps_b200.compression.manager import (add_sentinel, is_compressed_layer_names,
                                                    strip_sentinel)
from kvserve_hpdps_b200.compression.wire import CompressedWire, build_wire, restore_from_wire
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
        self._grouped_pending: dict[int, dict] = {}
        self._side_stream = None
        self._expected_msgs: dict[str, int] = {}
        self._rid2tid: dict[str, str] = {}
        self._pending_send_rids: set[str] = set()
        self._err_monitor = None
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
        for t in transfer_ids:
            if t in self._ctl_wait:
                self._ctl_done.append((t, latency_ms))
            stat = self._stats_wait.pop(t, None)
            if stat is not None:
                rid, orig, wire, ms, span = stat
                write_compression_stats(rid, t, orig, nbytes if nbytes else wire,
                                        compress_ms=ms, prefill_span_ms=span)

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
        if self._side_stream is not None and comp is not None and comp.supports_paged():
            ready = torch.cuda.current_stream().record_event()
            requests = [(rm.block_ids, len(rm.token_ids)) for rm in meta.requests]
            tids = [rm.transfer_id for rm in meta.requests]
            try:
                with torch.cuda.stream(self._side_stream):
                    self._side_stream.wait_event(ready)
                    # one grouped message for the layer; on the NVLink ring the
                    # producer kernels store it straight into the consumer's memory
                    comp.send_paged_requests(self._transport, tids[0], add_sentinel([layer_name]),
                                             [kv_layer], [layer_index(layer_name)], requests,
                                             member_tids=tids)
            except Exception:  # noqa: BLE001
                # as in the off mode: a compression failure sends this layer's raw
                # KV, one message per request (the consumer still counts one
                # message per layer for each transfer id)
                logger.exception("compression of %s failed; sending raw KV", layer_name)
                for rm in meta.requests:
                    raw = extract_kv_from_layer_by_blocks(kv_layer, rm.block_ids).unsqueeze(0)
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
            if comp is not None and comp.supports_paged() and layers[0].is_cuda:
                try:
                    with nvtx("kvs.compress_send"):
                        info = comp.send_paged_requests(
                            self._transport, tid, add_sentinel(names), layers,
                            [layer_index(n) for n in names], [(rm.block_ids, len(rm.token_ids))],
                            member_tids=[tid])
                except Exception:  # noqa: BLE001
                    # as the reference does: a compression failure sends the raw KV
                    logger.exception("compression of %s failed; sending raw KV", rid)
                    info = None
                if info is not None:
                    self._expected_msgs[tid] = 1
                    stat = (rid, info["original_size"], info["wire_nbytes"],
                            (time.monotonic() - t0) * 1e3, span)
                    if self._listening:  # written with the exact size once it is out
                        self._stats_wait[tid] = stat
                    else:
                        write_compression_stats(rid, tid, stat[1], stat[2], compress_ms=stat[3],
                                                prefill_span_ms=stat[4])
                    continue
                comp = None
            if comp is None and hasattr(self._transport, "send_paged") and layers[0].is_cuda:
                # raw KV: one gather launch from the paged caches into the peer ring
                with nvtx("kvs.send_raw"):
                    self._transport.send_paged(tid, names, layers, rm.block_ids)
                self._expected_msgs[tid] = 1
                continue
            stacked = torch.stack([extract_kv_from_layer_by_blocks(l, rm.block_ids)
                                   for l in layers], 0)
            cd = comp.compress(stacked, rid) if comp is not None else None
            if cd is not None:
                compress_ms = (time.monotonic() - t0) * 1e3
                if self._listening:  # completed by _apply_controller_feedback
                    self._ctl_wait[tid] = (rid, compress_ms, time.monotonic())
                nbytes = self._send_compressed(tid, names, cd)
                if not self._listening:
                    comp.update_controller(rid, (time.monotonic() - t0) * 1e3)
                write_compression_stats(rid, tid, stacked.numel() * stacked.element_size(), nbytes,
                                        compress_ms=(time.monotonic() - t0) * 1e3,
                                        prefill_span_ms=span)
            else:
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
        self._pending_send_rids -= done
        for rid in done:
            tid = self._rid2tid.pop(rid, None)
            if tid is not None:
                self._transport.clear_sent(tid)
                self._expected_msgs.pop(tid, None)
        return (done or None), None

    # ================================================================ consumer
    def start_load_kv(self, forward_context: Any, **kwargs: Any) -> None:
        if self.is_producer:
            return
        timeline("D load_enter")
        self._drain()
        meta = self._get_connector_metadata()
        if not isinstance(meta, CompressedKVConnectorMetadata):
            return
        streaming = self._overlap_mode == "stream" and self._num_layers > 0
        # one deadline for the step: with a dead producer the step returns
        # after LOAD_TIMEOUT_S, not after that long for each of its requests
        deadline = time.monotonic() + LOAD_TIMEOUT_S
        for rm in meta.requests:
            need = self._num_layers if streaming else 1
            got = 0
            while got < need:
                got += self._load_available(rm, forward_context)
                if got >= need:
                    break
                if time.monotonic() > deadline:
                    logger.warning("timeout loading KV of %s (transfer %s): %d/%d messages",
                                   rm.request_id, rm.transfer_id, got, need)
                    break
                waiter = getattr(self._transport, "wait_received", None)
                if waiter is not None:
                    waiter(0.002)  # wakes as soon as a message header arrives
                else:
                    time.sleep(0.002)
                self._drain()
        if torch.cuda.is_available() and meta.requests:
            # device-side failures of earlier loads (flag timeouts, checksum
            # mismatches, corrupt streams), read without waiting on the GPU
            if self._err_monitor is None:
                from kvserve_hpdps_b200.ops import kernels as K
                self._err_monitor = K.ErrorMonitor(torch.device("cuda", torch.cuda.current_device()))
            code = self._err_monitor.poll()
            if code:
                from kvserve_hpdps_b200.ops import kernels as K
                logger.error("device error %d (%s) while loading KV in an earlier step", code,
                             K.ERR_NAMES.get(code, "?"))
        timeline("D load_exit")

    def _drain(self) -> None:
        for tid, msgs in (self._transport.drain_received() or {}).items():
            for m in msgs:
                self._worker_received[tid].append(m)

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

    def _load_available(self, rm: ReqMeta, forward_context: Any) -> int:
        """Decode every message available for this request; returns how many
        messages were consumed."""
        q = self._worker_received.get(rm.transfer_id)
        n = 0
        while q:
            names, payload = q.popleft()
            n += 1
            if payload is None:
                logger.error("transport reported a failed transfer for %s", rm.request_id)
                continue
            try:
                self._inject(rm, names, payload, forward_context)
            except Exception as e:  # noqa: BLE001
                logger.error("decode of %s failed: %s", rm.request_id, e)
        if q is not None and not q:
            self._worker_received.pop(rm.transfer_id, None)
        return n

    def _inject(self, rm: ReqMeta, names: list[str], payload: Any, forward_context: Any) -> None:
        tr = self._transport
        dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() \
            else torch.device("cpu")
        if hasattr(tr, "prepare"):
            tr.prepare(payload, dev)
        if isinstance(payload, dict) and payload.get("__ring_raw__"):
            payload_t = payload["tensor"]
        else:
            payload_t = payload
        t0 = time.monotonic()
        try:
            with nvtx("kvs.inject"):
                self._inject_body(rm, names, payload, payload_t, forward_context, t0)
        finally:  # the ring space returns even when decoding fails
            if hasattr(tr, "release"):
                tr.release(payload, dev)

    def _inject_body(self, rm: ReqMeta, names: list[str], payload: Any, payload_t: Any,
                     forward_context: Any, t0: float) -> None:
        if is_compressed_layer_names(names):
            names = strip_sentinel(names)
            wire = CompressedWire(payload["meta"], payload["body_chunks"], payload["aux_tensors"])
            cd = restore_from_wire(wire)
            md = cd.metadata or {}
            comp = self._get_compressor()
            if md.get("layout") in ("items", "items_packed"):
                self._inject_items(rm, names, cd, comp, forward_context)
            else:
                kv = comp.decompress(cd)
                if kv is None:
                    raise RuntimeError("decompression returned None")
                for i, name in enumerate(names):
                    cache = self._layer_cache(name, forward_context)
                    if cache is not None:
                        inject_kv_into_layer_by_blocks(cache, kv[i], rm.block_ids, rm.request_id)
            write_decode_stats(rm.request_id, rm.transfer_id, (time.monotonic() - t0) * 1e3)
        else:
            caches = [self._layer_cache(n, forward_context) for n in names]
            if self._scatter_raw(rm, caches, payload, payload_t):
                return
            for cache, part in zip(caches, payload_t):
                if cache is not None:
                    inject_kv_into_layer_by_blocks(cache, part, rm.block_ids, rm.request_id)

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

    def _inject_items(self, rm: ReqMeta, names: list[str], cd, comp, forward_context) -> None:
        """Fused message (one or more requests x layers): decode into the
        registered caches at this request's blocks."""
        md = cd.metadata
        tids = md["member_tids"]
        caches = [self._layer_cache(n, forward_context) for n in names]
        if any(c is None for c in caches):
            raise RuntimeError("missing KV cache tensor for a layer of the message")
        if len(tids) == 1:
            comp.decompress_paged_requests(cd, caches, [(rm.block_ids, md["member_tokens"][0])])
            return
        # grouped: decode the members scheduled now; keep the rest for later
        key = id(cd.compressed_tensor)
        entry = self._grouped_pending.setdefault(key, {"cd": cd, "names": names, "left": set(tids)})
        meta = self._get_connector_metadata()
        here = {r.transfer_id: r for r in meta.requests} if meta is not None else {}
        reqs = []
        for i, t in enumerate(tids):
            r = here.get(t)
            reqs.append((r.block_ids, md["member_tokens"][i]) if r is not None and t in entry["left"]
                        else (None, md["member_tokens"][i]))
        sub = [(i, b) for i, (b, _) in enumerate(reqs) if b is not None]
        if sub:
            comp.manager.decompress_members(cd, caches, {i: b for i, b in sub})
            for i, _ in sub:
                entry["left"].discard(tids[i])
        if not entry["left"]:
            self._grouped_pending.pop(key, None)

    def wait_for_layer_load(self, layer_name: str) -> None:
        return None

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
