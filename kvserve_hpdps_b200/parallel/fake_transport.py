"""In-process transport pair for tests (no sockets, no devices required).

``FakeTransportPair.producer()`` / ``.consumer()`` implement the transport
API; messages are cloned into the consumer's inbox in send order.  Failure
injection on the host: ``drop_next`` silently drops the next message (the
producer counts it as sent), ``refuse_next`` delivers the FAILED sentinel
(as a consumer that could not allocate; the producer counts it in
``failed_layers``, as the refusing ACK would tell it), ``delay_s`` delays
delivery on a timer thread.
"""

from __future__ import annotations

import threading
from collections import defaultdict, deque
from typing import Any, Optional

import torch

from kvserve_hpdps_b200.parallel.control import notify_sent
from kvserve_hpdps_b200.parallel.nccl_transport import FAILED_LAYER_NAMES, FAILED_PAYLOAD
from kvserve_hpdps_b200.utils.logger import get_logger

logger = get_logger(__name__)


class FakeTransportPair:
    def __init__(self):
        self.lock = threading.Lock()
        self.inbox: dict[str, deque] = defaultdict(deque)
        self.sent: dict[str, int] = defaultdict(int)
        self.failed: dict[str, int] = defaultdict(int)
        self.listeners: list = []
        self.drop_next = 0
        self.refuse_next = 0
        self.delay_s = 0.0
        self.messages = 0

    def producer(self) -> "_FakeEnd":
        return _FakeEnd(self, True)

    def consumer(self) -> "_FakeEnd":
        return _FakeEnd(self, False)


class _FakeEnd:
    def __init__(self, pair: FakeTransportPair, is_sender: bool):
        self.pair = pair
        self.is_sender = is_sender

    def _deliver(self, rid: str, item) -> bool:
        """Queue a message for the consumer; False when it was refused."""
        p = self.pair
        with p.lock:
            p.messages += 1
            if p.drop_next > 0:
                p.drop_next -= 1
                return True
            if p.refuse_next > 0:
                p.refuse_next -= 1
                item = (FAILED_LAYER_NAMES, FAILED_PAYLOAD)
                refused = True
            else:
                refused = False

        def put():
            with p.lock:
                p.inbox[rid].append(item)

        if p.delay_s > 0:
            threading.Timer(p.delay_s, put).start()
        else:
            put()
        return not refused

    def send(self, request_id: str, layer_names: list[str], stacked_kv: torch.Tensor) -> None:
        ok = self._deliver(request_id, (list(layer_names), stacked_kv.clone()))
        self._count_sent(None, request_id, ok, stacked_kv.numel() * stacked_kv.element_size())

    def _count_sent(self, member_tids: Optional[list[str]], request_id: str,
                    ok: bool = True, nbytes: int = 0) -> None:
        """A message without member ids counts for its request id; listeners
        hear of accepted messages with their size in bytes."""
        table = self.pair.sent if ok else self.pair.failed
        with self.pair.lock:
            for t in (member_tids or [request_id]):
                table[t] += 1
        if ok:
            notify_sent(self.pair.listeners, request_id, list(member_tids or [request_id]),
                        self.pair.delay_s * 1e3, int(nbytes), logger)

    def send_bundle(self, request_id, layer_names, meta, body_chunks, aux_tensors,
                    member_tids: Optional[list[str]] = None) -> None:
        payload = {"__bundle__": True, "meta": meta,
                   "body_chunks": [t.clone() for t in body_chunks],
                   "aux_tensors": [t.clone() for t in aux_tensors]}
        ok = self._deliver(request_id, (list(layer_names), payload))
        self._count_sent(member_tids, request_id, ok,
                         sum(t.numel() * t.element_size() for t in body_chunks)
                         + sum(t.numel() * t.element_size() for t in aux_tensors))

    def sent_layers(self, tid: str) -> int:
        with self.pair.lock:
            return self.pair.sent.get(tid, 0)

    def add_sent_listener(self, fn) -> None:
        """``fn(request_id, transfer_ids, latency_ms)`` for every message the
        consumer accepted (latency: the injected delay)."""
        self.pair.listeners.append(fn)

    def failed_layers(self, tid: str) -> int:
        with self.pair.lock:
            return self.pair.failed.get(tid, 0)

    def clear_sent(self, tid: str) -> None:
        with self.pair.lock:
            self.pair.sent.pop(tid, None)
            self.pair.failed.pop(tid, None)

    def wait_for_sent(self, timeout_s: Optional[float] = None) -> bool:
        return True

    def drain_received(self) -> dict[str, list[tuple[list[str], Any]]]:
        with self.pair.lock:
            out = {k: list(v) for k, v in self.pair.inbox.items() if v}
            self.pair.inbox.clear()
        return out

    def close(self) -> None:
        return None
