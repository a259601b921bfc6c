"""Point-to-point transport over a torch process group (NCCL; gloo for CPU tests).

Public API of the reference transport (kvserve_v1/transport/nccl_transport.py:54-462):

* producer: ``send(request_id, layer_names, stacked_kv)``,
  ``send_bundle(request_id, layer_names, meta, body_chunks, aux_tensors,
  member_tids=None)``, ``sent_layers(tid)``, ``clear_sent(tid)``,
  ``wait_for_sent()``; ``failed_layers(tid)`` (new) counts the messages the
  consumer refused or that could not be sent, so that a caller that frees a
  request's blocks once its messages are out does not wait for them forever;
  ``add_sent_listener(fn)`` (new) calls ``fn(request_id, transfer_ids,
  latency_ms)`` on the send thread when a message has left, with the time
  from its ``send``/``send_bundle`` call;
* consumer: ``drain_received() -> {transfer_id: [(layer_names, payload)]}``
  where payload is a tensor (raw), a bundle dict (``{"__bundle__": True,
  "meta", "body_chunks", "aux_tensors"}``) or ``FAILED_PAYLOAD`` (None) when
  the consumer refused the message (allocation failure, no channel).

Protocol per message: the producer's send thread sends a ``PUT`` /
``PUT_BUNDLE`` header over the ZMQ channel and waits for the consumer's ACK;
the consumer allocates the tensors, ACKs, and posts the receives; the
producer then posts its sends.  The consumer only posts receives after a
header, so no receive is pending while the engine captures CUDA graphs.

Every header gets an answer: the consumer refuses (``b"1"``) a header it
cannot read or allocate for, and an unknown command, so a producer never
waits out its timeout on a live consumer.  A producer whose request timed
out cannot tell whether the consumer accepted it and posted receives, and
the next message's tensors could then be matched with those receives, so
after a control timeout the producer refuses every later send at once
(``ctl_failed``; logged) and the pair needs a new transport.

The 2-rank process group is built from a TCPStore the consumer hosts on
``kv_port + tp_rank + STORE_PORT_OFFSET`` (producer rank 0, consumer rank 1).
This transport is the baseline and the fallback of the NVLink ring transport
(``p2p_transport.py``), e.g. across nodes.
"""

from __future__ import annotations

import datetime
import threading
import time
from collections import defaultdict, deque
from typing import Any, Optional

import torch

from kvserve_hpdps_b200.parallel.control import (ACK_OK, ACK_REFUSED, ConsumerChannel,
                                                 ProducerChannel, channel_port, notify_sent)
from kvserve_hpdps_b200.utils.logger import get_logger
from kvserve_hpdps_b200.utils.stats import write_transfer_stats

logger = get_logger(__name__)

FAILED_PAYLOAD: Any = None
FAILED_LAYER_NAMES: list[str] = []
STORE_PORT_OFFSET = 1000


def tensor_spec(t: torch.Tensor) -> dict[str, Any]:
    return {"shape": list(t.shape), "dtype": str(t.dtype).replace("torch.", "")}


def alloc_from_spec(spec: dict[str, Any], device: torch.device) -> torch.Tensor:
    return torch.empty(tuple(spec["shape"]), dtype=getattr(torch, spec["dtype"]), device=device)


def make_pair_group(host: str, port: int, rank: int, backend: str, timeout_s: float = 120.0):
    """2-rank process group over a TCPStore (rank 1 hosts the store)."""
    import torch.distributed as dist
    store = dist.TCPStore(host if rank == 0 else "0.0.0.0", port, 2, rank == 1,
                          timeout=datetime.timedelta(seconds=timeout_s))
    if backend == "nccl":
        pg = dist.ProcessGroupNCCL(store, rank, 2)
    else:
        pg = dist.ProcessGroupGloo(store, rank, 2, datetime.timedelta(seconds=timeout_s))
    return pg, store


def _deferred_codec(meta: Any) -> Optional[str]:
    inner = meta.get("metadata") if isinstance(meta, dict) else None
    return inner.get("deferred_codec") if isinstance(inner, dict) else None


def _encode_deferred(meta: dict, body: list[torch.Tensor],
                     device: torch.device) -> tuple[dict, list[torch.Tensor]]:
    """Entropy-code a message body the producer left as plain codes
    (``deferred_codec`` in its metadata) and return the wire metadata and
    body of the coded message: the 16-byte container header and the stream,
    trimmed to the stream's own length (read back here, off the engine
    thread).  The consumer then decodes it like any coded body."""
    from kvserve_hpdps_b200.compression.codec import encode_bytes
    inner = dict(meta["metadata"])
    codec = inner.pop("deferred_codec")
    inner.pop("container", None)
    codes = torch.cat([t.contiguous().view(torch.uint8).reshape(-1) for t in body]) \
        if len(body) > 1 else body[0].contiguous().view(torch.uint8).reshape(-1)
    if device.type == "cuda":
        with torch.cuda.device(device):
            stream = torch.cuda.current_stream(device)
            coded = encode_bytes(codes, codec)  # reads the size back: a sync on this thread
            stream.synchronize()
    else:
        coded = encode_bytes(codes, codec)
    out = dict(meta)
    out["metadata"] = inner
    out["body_mode"] = "single"
    out["body_spec"] = tensor_spec(coded)
    out["compressed_size"] = int(coded.numel())
    return out, [coded]


class NcclTransport:
    def __init__(self, is_sender: bool, host: str, port: int, local_rank: int = 0,
                 channel_rank: int = 0, backend: str = "nccl", timeout_s: float = 60.0):
        self.is_sender = is_sender
        self.backend = backend
        self.port = channel_port(port, channel_rank)
        self.store_port = self.port + STORE_PORT_OFFSET
        self.host = host
        self.timeout_s = timeout_s
        self.device = torch.device("cuda", local_rank) if backend == "nccl" else torch.device("cpu")
        self._pg = None
        self._closed = False
        if is_sender:
            self._ctl = ProducerChannel(host, self.port, timeout_s)
            self._ctl.send({"cmd": "INIT", "backend": backend, "store_port": self.store_port})
            self._pg, self._store = make_pair_group(host, self.store_port, 0, backend)
            self._cv = threading.Condition()
            self._queue: deque = deque()
            self._inflight = 0
            self._sent_lock = threading.Lock()
            self._sent: dict[str, int] = defaultdict(int)
            self._failed: dict[str, int] = defaultdict(int)
            self._listeners: list = []
            self.ctl_failed = False
            self._thread = threading.Thread(target=self._send_loop, daemon=True,
                                            name="kvs-send")
            self._thread.start()
        else:
            self._ctl = ConsumerChannel(self.port)
            self._lock = threading.Lock()
            self._received: dict[str, deque] = defaultdict(deque)
            self._thread = threading.Thread(target=self._listen_loop, daemon=True,
                                            name="kvs-listen")
            self._thread.start()

    # ------------------------------------------------------------ producer
    def _ready_event(self):
        if self.device.type == "cuda":
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            return ev
        return None

    def send(self, request_id: str, layer_names: list[str], stacked_kv: torch.Tensor) -> None:
        assert self.is_sender
        t = stacked_kv.to(self.device).contiguous()
        with self._cv:
            self._queue.append(("tensor", request_id, list(layer_names), t, self._ready_event(), None,
                                time.monotonic()))
            self._cv.notify()

    def send_bundle(self, request_id: str, layer_names: list[str], meta: dict,
                    body_chunks: list[torch.Tensor], aux_tensors: list[torch.Tensor],
                    member_tids: Optional[list[str]] = None) -> None:
        assert self.is_sender
        body = [t.to(self.device).contiguous() for t in body_chunks]
        aux = [t.to(self.device).contiguous() for t in aux_tensors]
        with self._cv:
            self._queue.append(("bundle", request_id, list(layer_names), (meta, body, aux),
                                self._ready_event(), member_tids, time.monotonic()))
            self._cv.notify()

    def sent_layers(self, transfer_id: str) -> int:
        with self._sent_lock:
            return self._sent.get(transfer_id, 0)

    def add_sent_listener(self, fn) -> None:
        """``fn(request_id, transfer_ids, latency_ms)`` after each message left
        (with an ``nbytes`` keyword, when it takes one: the bytes sent)."""
        self._listeners.append(fn)

    def failed_layers(self, transfer_id: str) -> int:
        with self._sent_lock:
            return self._failed.get(transfer_id, 0)

    def _count(self, table: dict, request_id: str, member_tids) -> None:
        with self._sent_lock:  # a message without member ids counts for its request id
            for tid in (member_tids or [request_id]):
                table[tid] += 1

    def clear_sent(self, transfer_id: str) -> None:
        with self._sent_lock:
            self._sent.pop(transfer_id, None)
            self._failed.pop(transfer_id, None)

    def wait_for_sent(self, timeout_s: Optional[float] = None) -> bool:
        deadline = None if timeout_s is None else time.monotonic() + timeout_s
        with self._cv:
            while self._queue or self._inflight:
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    return False
                self._cv.wait(timeout=left if left is not None else 1.0)
        return True

    def _send_loop(self) -> None:
        while not self._closed:
            with self._cv:
                while not self._queue and not self._closed:
                    self._cv.wait(timeout=0.5)
                if self._closed:
                    return
                item = self._queue.popleft()
                self._inflight += 1
            try:
                if not self._send_item(*item):
                    self._count(self._failed, item[1], item[5])
            except Exception as e:  # noqa: BLE001
                logger.error("send of %s failed: %s", item[1], e)
                self._count(self._failed, item[1], item[5])
            finally:
                with self._cv:
                    self._inflight -= 1
                    self._cv.notify_all()

    def _p2p_send(self, tensors: list[torch.Tensor]) -> None:
        works = [self._pg.send([t], 1, 0) for t in tensors if t.numel() > 0]
        for w in works:
            w.wait()
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()

    def _send_item(self, kind, request_id, layer_names, payload, event, member_tids,
                   t_enqueued: float) -> bool:
        """One message; False when it was refused or not sent."""
        if kind == "tensor":
            t = payload
            msg = {"cmd": "PUT", "request_id": request_id, "layer_names": layer_names,
                   **tensor_spec(t)}
            tensors = [t]
        else:
            meta, body, aux = payload
            if _deferred_codec(meta) is not None:
                # codes left for the transport to encode: encode them here, on the
                # send thread, and send only the stream's own bytes
                if event is not None:
                    event.synchronize()
                    event = None
                meta, body = _encode_deferred(meta, body, self.device)
            msg = {"cmd": "PUT_BUNDLE", "request_id": request_id, "layer_names": layer_names,
                   "meta": meta, "body_specs": [tensor_spec(t) for t in body],
                   "aux_specs": [tensor_spec(t) for t in aux]}
            tensors = body + aux
        if self.ctl_failed:
            logger.error("control channel failed earlier; %s not sent", request_id)
            return False
        stale = self._ctl.discard_pending()
        if stale:
            logger.warning("dropped %d stale control replies", stale)
        ack = self._ctl.request(msg, self.timeout_s)
        if ack is None:
            self.ctl_failed = True
            logger.error("no answer to %s within %.1f s: the pair's message order can no longer "
                         "be trusted, later sends are refused", request_id, self.timeout_s)
            return False
        if ack != ACK_OK:
            logger.error("consumer refused %s (%r)", request_id, ack)
            return False
        if event is not None:
            event.synchronize()
        t0 = time.monotonic()
        self._p2p_send(tensors)
        nbytes = sum(t.numel() * t.element_size() for t in tensors)
        self._count(self._sent, request_id, member_tids)
        now = time.monotonic()
        write_transfer_stats(request_id, (now - t0) * 1e3, nbytes,
                             transport="nccl" if self.backend == "nccl" else self.backend)
        notify_sent(self._listeners, request_id, list(member_tids or [request_id]),
                    (now - t_enqueued) * 1e3, nbytes, logger)
        return True

    # ------------------------------------------------------------ consumer
    def drain_received(self) -> dict[str, list[tuple[list[str], Any]]]:
        assert not self.is_sender
        with self._lock:
            out = {k: list(v) for k, v in self._received.items() if v}
            self._received.clear()
        return out

    def _mark_failed(self, request_id: str) -> None:
        with self._lock:
            self._received[request_id].append((FAILED_LAYER_NAMES, FAILED_PAYLOAD))

    def _recv(self, tensors: list[torch.Tensor]) -> None:
        works = [self._pg.recv([t], 0, 0) for t in tensors if t.numel() > 0]
        for w in works:
            w.wait()
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()

    def _listen_loop(self) -> None:
        while not self._closed:
            try:
                got = self._ctl.poll(200)
                if got is None:
                    continue
                ident, msg = got
                cmd = msg.get("cmd")
                if cmd == "INIT":
                    self._pg, self._store = make_pair_group("0.0.0.0", msg["store_port"], 1,
                                                            msg.get("backend", self.backend))
                    continue
                if cmd not in ("PUT", "PUT_BUNDLE"):
                    self._handle_extra(ident, msg)
                    continue
                rid = msg.get("request_id")
                if not isinstance(rid, str) or not isinstance(msg.get("layer_names"), list):
                    logger.error("malformed %s header refused", cmd)
                    self._ctl.reply(ident, ACK_REFUSED)
                    if isinstance(rid, str):
                        self._mark_failed(rid)
                    continue
                if self._pg is None:
                    self._ctl.reply(ident, ACK_REFUSED)
                    self._mark_failed(rid)
                    continue
                try:
                    if cmd == "PUT":
                        tensors = [alloc_from_spec(msg, self.device)]
                    else:
                        body = [alloc_from_spec(s, self.device) for s in msg["body_specs"]]
                        aux = [alloc_from_spec(s, self.device) for s in msg["aux_specs"]]
                        tensors = body + aux
                except (torch.cuda.OutOfMemoryError, RuntimeError, KeyError, TypeError,
                        ValueError, AttributeError) as e:
                    logger.error("allocation for %s failed: %s", rid, e)
                    self._ctl.reply(ident, ACK_REFUSED)
                    self._mark_failed(rid)
                    continue
                self._ctl.reply(ident, ACK_OK)
                self._recv(tensors)
                payload = tensors[0] if cmd == "PUT" else {
                    "__bundle__": True, "meta": msg["meta"], "body_chunks": body,
                    "aux_tensors": aux}
                with self._lock:
                    self._received[rid].append((msg["layer_names"], payload))
            except Exception as e:  # noqa: BLE001
                logger.error("listener error: %s", e)

    def _handle_extra(self, ident: bytes, msg: dict) -> None:
        """Unknown or undecodable message: refused, so a sender waiting for
        an answer gets one (a sender that expects none drops it before its
        next request)."""
        logger.warning("unknown control message %r%s", msg.get("cmd"),
                       f" ({msg['error']})" if msg.get("error") else "")
        self._ctl.reply(ident, ACK_REFUSED)

    def close(self) -> None:
        self._closed = True
        try:
            self._ctl.close()
        except Exception:  # noqa: BLE001
            pass
