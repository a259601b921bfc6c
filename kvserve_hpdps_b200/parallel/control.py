"""ZMQ control channel between a producer and a consumer rank.

One channel per TP rank on ``kv_port + tp_rank`` (reference:
kvserve_v1/transport/nccl_transport.py:61-130): the consumer binds a ROUTER,
the producer connects a DEALER whose identity is ``host:port``.  Messages are
msgpack dicts with a ``cmd`` field; the reference's verbs ``INIT``, ``PUT``
and ``PUT_BUNDLE`` (and its one-byte ACKs ``b"0"`` ok / ``b"1"`` refused)
keep their meaning, and this framework adds ``RING_MAP`` (receive-ring
handles), ``PUT_RING`` (a payload written into the ring by the producer's
kernels) and ``FREE`` (ring space returned by the consumer).

All receives take a timeout so no thread blocks forever on a dead peer.
"""

from __future__ import annotations

import threading
from typing import Any, Optional

import msgpack
import zmq

ACK_OK = b"0"
ACK_REFUSED = b"1"


def channel_port(kv_port: int, tp_rank: int) -> int:
    return int(kv_port) + int(tp_rank)


def pack(msg: dict[str, Any]) -> bytes:
    return msgpack.dumps(msg, use_bin_type=True)


def unpack(raw: bytes) -> dict[str, Any]:
    return msgpack.loads(raw, raw=False)


class ProducerChannel:
    """DEALER side.  ``request`` sends a message and waits for the reply."""

    def __init__(self, host: str, port: int, timeout_s: float = 60.0):
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.DEALER)
        self.sock.setsockopt_string(zmq.IDENTITY, f"{host}:{port}:{id(self)}")
        self.sock.setsockopt(zmq.LINGER, 0)
        self.sock.connect(f"tcp://{host}:{port}")
        self.timeout_ms = int(timeout_s * 1000)
        self.lock = threading.Lock()

    def send(self, msg: dict[str, Any]) -> None:
        with self.lock:
            self.sock.send(pack(msg))

    def enable_wakeup(self) -> None:
        """Let other threads interrupt :meth:`recv_or_wake` (an inproc pair):
        a thread that owns the socket can then sleep in a long poll and still
        send a queued message the moment it is queued."""
        addr = f"inproc://kvs-wake-{id(self)}"
        self._wake_rx = self.ctx.socket(zmq.PAIR)
        self._wake_rx.setsockopt(zmq.LINGER, 0)
        self._wake_rx.bind(addr)
        self._wake_tx = self.ctx.socket(zmq.PAIR)
        self._wake_tx.setsockopt(zmq.LINGER, 0)
        self._wake_tx.connect(addr)
        self._wake_lock = threading.Lock()
        self._poller = zmq.Poller()
        self._poller.register(self.sock, zmq.POLLIN)
        self._poller.register(self._wake_rx, zmq.POLLIN)

    def wake(self) -> None:
        """Interrupt the owner thread's :meth:`recv_or_wake` (any thread)."""
        with self._wake_lock:
            try:
                self._wake_tx.send(b"", zmq.NOBLOCK)
            except zmq.Again:  # already woken many times: it will look anyway
                pass

    def recv_or_wake(self, timeout_s: float) -> Optional[bytes]:
        """A message from the peer, or None after ``timeout_s`` or a
        :meth:`wake` (owner thread only)."""
        events = dict(self._poller.poll(int(timeout_s * 1000)))
        if self._wake_rx in events:
            while True:
                try:
                    self._wake_rx.recv(zmq.NOBLOCK)
                except zmq.Again:
                    break
        if self.sock in events:
            return self.sock.recv()
        return None

    def recv(self, timeout_s: Optional[float] = None) -> Optional[bytes]:
        t = self.timeout_ms if timeout_s is None else int(timeout_s * 1000)
        if self.sock.poll(t, zmq.POLLIN):
            return self.sock.recv()
        return None

    def discard_pending(self) -> int:
        """Drop replies already queued on the socket (a late answer to a
        request that timed out) so that the next ``request`` reads its own
        reply; returns how many were dropped.  Only for channels whose every
        incoming message is a reply."""
        n = 0
        with self.lock:
            while self.sock.poll(0, zmq.POLLIN):
                self.sock.recv()
                n += 1
        return n

    def request(self, msg: dict[str, Any], timeout_s: Optional[float] = None) -> Optional[bytes]:
        with self.lock:
            self.sock.send(pack(msg))
            t = self.timeout_ms if timeout_s is None else int(timeout_s * 1000)
            if self.sock.poll(t, zmq.POLLIN):
                return self.sock.recv()
        return None

    def close(self) -> None:
        self.sock.close(0)
        for name in ("_wake_rx", "_wake_tx"):
            sock = getattr(self, name, None)
            if sock is not None:
                sock.close(0)


class ConsumerChannel:
    """ROUTER side.  ``poll`` returns (identity, message) or None."""

    def __init__(self, port: int, bind_host: str = "*"):
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.ROUTER)
        self.sock.setsockopt(zmq.LINGER, 0)
        self.sock.bind(f"tcp://{bind_host}:{port}")
        self.lock = threading.Lock()

    def poll(self, timeout_ms: int = 100) -> Optional[tuple[bytes, dict[str, Any]]]:
        """(identity, message); a frame that is not a msgpack dict comes back
        as ``{"cmd": None, "error": ...}`` so that the caller can refuse it
        instead of leaving the sender waiting for a reply."""
        if self.sock.poll(timeout_ms, zmq.POLLIN):
            frames = self.sock.recv_multipart()
            try:
                msg = unpack(frames[-1])
            except Exception as e:  # noqa: BLE001 - any decode failure
                return frames[0], {"cmd": None, "error": f"undecodable frame: {e}"}
            if not isinstance(msg, dict):
                return frames[0], {"cmd": None, "error": f"not a dict: {type(msg).__name__}"}
            return frames[0], msg
        return None

    def reply(self, identity: bytes, payload: bytes) -> None:
        with self.lock:
            self.sock.send_multipart([identity, payload])

    def close(self) -> None:
        self.sock.close(0)


def _takes_nbytes(fn) -> bool:
    import inspect
    try:
        params = inspect.signature(fn).parameters.values()
    except (TypeError, ValueError):
        return False
    return any(p.name == "nbytes" or p.kind == p.VAR_KEYWORD for p in params)


def notify_sent(listeners, request_id: str, transfer_ids: list, latency_ms: float,
                nbytes: int, log) -> None:
    """Call every sent listener ``fn(request_id, transfer_ids, latency_ms)``;
    listeners that accept an ``nbytes`` keyword also get the bytes that
    crossed the link.  A failing listener is logged, not raised."""
    for fn in list(listeners):
        try:
            if _takes_nbytes(fn):
                fn(request_id, list(transfer_ids), latency_ms, nbytes=nbytes)
            else:
                fn(request_id, list(transfer_ids), latency_ms)
        except Exception as e:  # noqa: BLE001
            log.error("sent listener failed: %s", e)
