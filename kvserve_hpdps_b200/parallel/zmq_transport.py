"""Legacy host-memory transport: PUSH/PULL of CPU tensors over ZMQ.

Kept for parity with the reference's unused legacy path
(kvserve_v1/transport/zmq_transport.py:20-95) and for machines without a GPU
data path: the producer pushes ``[header, tensor bytes]``; a consumer thread
pulls and buffers ``{request_id: (layer_names, tensor)}``.  Tensors travel as
raw bytes with a dtype/shape header (no pickle).
"""

from __future__ import annotations

import threading

import msgpack
import torch
import zmq

from kvserve_hpdps_b200.utils.logger import get_logger

logger = get_logger(__name__)


class ZmqTransport:
    def __init__(self, is_sender: bool, host: str, port: int):
        self.is_sender = is_sender
        self._ctx = zmq.Context.instance()
        if is_sender:
            self._sock = self._ctx.socket(zmq.PUSH)
            self._sock.setsockopt(zmq.LINGER, 1000)
            self._sock.connect(f"tcp://{host}:{port}")
        else:
            self._sock = self._ctx.socket(zmq.PULL)
            self._sock.bind(f"tcp://*:{port}")
            self._lock = threading.Lock()
            self._received: dict[str, tuple[list[str], torch.Tensor]] = {}
            self._closed = False
            self._thread = threading.Thread(target=self._recv_loop, daemon=True, name="kvs-zmq")
            self._thread.start()

    def send(self, request_id: str, layer_names: list[str], stacked_kv: torch.Tensor) -> None:
        t = stacked_kv.detach().to("cpu").contiguous()
        hdr = msgpack.dumps({"request_id": request_id, "layer_names": list(layer_names),
                             "shape": list(t.shape), "dtype": str(t.dtype).replace("torch.", "")})
        self._sock.send_multipart([hdr, t.view(torch.uint8).numpy().tobytes()])

    def wait_for_sent(self) -> None:
        return None

    def drain_received(self) -> dict[str, tuple[list[str], torch.Tensor]]:
        with self._lock:
            out = dict(self._received)
            self._received.clear()
        return out

    def _recv_loop(self) -> None:
        while not self._closed:
            try:
                if not self._sock.poll(200, zmq.POLLIN):
                    continue
                hdr_raw, body = self._sock.recv_multipart()
                hdr = msgpack.loads(hdr_raw, raw=False)
                dtype = getattr(torch, hdr["dtype"])
                t = torch.frombuffer(bytearray(body), dtype=torch.uint8).view(dtype).reshape(hdr["shape"])
                with self._lock:
                    self._received[hdr["request_id"]] = (hdr["layer_names"], t)
            except Exception as e:  # noqa: BLE001
                logger.error("zmq recv error: %s", e)

    def close(self) -> None:
        if not self.is_sender:
            self._closed = True
        self._sock.close(0)
