"""NVLink receive-ring transport: producer kernels store into the consumer's memory.

Same public API as the NCCL transport (``send``, ``send_bundle``,
``sent_layers``, ``clear_sent``, ``wait_for_sent``, ``drain_received``) plus
two consumer hooks the connector calls around decoding:
``prepare(payload, device)`` launches a bounded device wait on the payload's
ready flag, ``release(payload, device)`` returns the payload's ring space once
the work queued on the stream so far has finished.

Design (one channel per TP rank, on ``kv_port + tp_rank``):

* the consumer owns a receive ring allocated with cudaMalloc (so its CUDA
  IPC handle names exactly the ring) followed by a table of ready flags;
  the producer asks for it with ``RING_HELLO`` and maps it with
  ``cudaIpcOpenMemHandle``;
* the producer allocates ring space itself (first-fit free list over the
  consumer's ring); the consumer returns space with ``FREE`` messages, so a
  message costs no round trip;
* a send enqueues one gather-copy kernel on the producer's transfer stream:
  every tensor of the message is stored into the peer ring over NVLink and
  the last CTA publishes the message's sequence number into its flag slot
  (``__threadfence_system`` + ``st.release.sys``); the ``PUT_RING`` header
  (tensor specs and ring offsets) goes over ZMQ right after the launch;
* the consumer wraps ring slices as tensors (``__cuda_array_interface__``,
  zero copy) and its decode kernels run after a bounded device wait on the
  flag (``ERR_FLAG_TIMEOUT`` instead of a hang if the producer died).

No TMA multicast and no library kernel reads the peer ring: only this
framework's own store loop writes it and its own kernels read the local copy.
"""

from __future__ import annotations

import queue
import threading
import time
from collections import defaultdict, deque
from dataclasses import dataclass
from typing import Any, Optional

import torch

from kvserve_hpdps_b200.parallel.control import (ConsumerChannel, ProducerChannel, channel_port,
                                                 notify_sent, pack, unpack)
from kvserve_hpdps_b200.parallel.nccl_transport import FAILED_LAYER_NAMES, FAILED_PAYLOAD
from kvserve_hpdps_b200.utils.logger import get_logger
from kvserve_hpdps_b200.utils.stats import write_transfer_stats

logger = get_logger(__name__)

ALIGN = 256
FLAG_STRIDE = 16


def _timing_event(stream) -> torch.cuda.Event:
    """An event with timing enabled, recorded on ``stream`` now."""
    ev = torch.cuda.Event(enable_timing=True)
    ev.record(stream)
    return ev


def _align(x: int) -> int:
    return (x + ALIGN - 1) // ALIGN * ALIGN


@dataclass
class RingMessage:
    """Ring space of one message being written by producer kernels."""
    base: int              # ring offset of the message
    total: int             # reserved bytes (tensors, alignment, checksum trailer)
    seq: int
    slot: int              # ready-flag slot
    offsets: list          # offset of each tensor inside the message
    sizes: list            # bytes of each tensor
    ptrs: list             # device address (consumer memory) of each tensor
    trailer_ptr: int       # where the finished checksum goes
    trailer_off: int       # its ring offset
    ck: torch.Tensor       # int64[2] checksum accumulators (producer memory)
    flag_ptr: int
    flag_value: int
    t0: Any                # timing event recorded before the message's first kernel


class RingAllocator:
    """First-fit free-list allocator over [0, capacity) (producer side)."""

    def __init__(self, capacity: int):
        self.capacity = int(capacity)
        self.free: list[tuple[int, int]] = [(0, self.capacity)]  # sorted (off, size)
        self.cv = threading.Condition()

    def try_alloc(self, size: int) -> Optional[int]:
        size = _align(size)
        for i, (off, sz) in enumerate(self.free):
            if sz >= size:
                if sz == size:
                    self.free.pop(i)
                else:
                    self.free[i] = (off + size, sz - size)
                return off
        return None

    def alloc(self, size: int, timeout_s: float) -> Optional[int]:
        deadline = time.monotonic() + timeout_s
        with self.cv:
            while True:
                off = self.try_alloc(size)
                if off is not None:
                    return off
                left = deadline - time.monotonic()
                if left <= 0:
                    return None
                self.cv.wait(timeout=min(left, 0.1))

    def release(self, off: int, size: int) -> bool:
        """Return [off, off + size) to the free list; a range that overlaps
        free space (a region returned twice) is refused and logged, so the
        list never hands the same bytes to two messages."""
        size = _align(size)
        with self.cv:
            if off < 0 or off + size > self.capacity or any(
                    o < off + size and off < o + s for o, s in self.free):
                logger.error("p2p: ring region [%d, %d) returned twice or out of range; ignored",
                             off, off + size)
                return False
            self.free.append((off, size))
            self.free.sort()
            merged = []
            for o, s in self.free:
                if merged and merged[-1][0] + merged[-1][1] == o:
                    merged[-1] = (merged[-1][0], merged[-1][1] + s)
                else:
                    merged.append((o, s))
            self.free = merged
            self.cv.notify_all()
        return True

    def free_bytes(self) -> int:
        with self.cv:
            return sum(s for _, s in self.free)


class _CudaView:
    """Zero-copy tensor view of raw device memory (__cuda_array_interface__)."""

    _TYPESTR = {torch.uint8: "|u1", torch.int8: "|i1", torch.int16: "<i2", torch.int32: "<i4",
                torch.int64: "<i8", torch.float16: "<f2", torch.float32: "<f4",
                torch.float64: "<f8"}

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (int(nbytes),), "typestr": "|u1",
                                         "data": (int(ptr), False), "version": 3}


def tensor_view(ptr: int, nbytes: int, dtype: torch.dtype, shape, device: int) -> torch.Tensor:
    if nbytes == 0:
        return torch.empty(shape, dtype=dtype, device=f"cuda:{device}")
    raw = torch.as_tensor(_CudaView(ptr, nbytes), device=f"cuda:{device}")
    return raw.view(dtype).reshape(shape)


class P2PTransport:
    def __init__(self, is_sender: bool, host: str, port: int, local_rank: int = 0,
                 channel_rank: int = 0, ring_bytes: int = 2 << 30, n_flags: int = 4096,
                 timeout_s: float = 60.0, flag_timeout_s: float = 30.0):
        self.is_sender = is_sender
        self.port = channel_port(port, channel_rank)
        self.device = torch.device("cuda", local_rank)
        self.local_rank = local_rank
        self.timeout_s = timeout_s
        self.flag_timeout_s = flag_timeout_s
        self._closed = False
        self._outbox: queue.Queue = queue.Queue()
        if is_sender:
            self._ctl = ProducerChannel(host, self.port, timeout_s)
            self._ctl.enable_wakeup()
            reply = self._ctl.request({"cmd": "RING_HELLO", "device": local_rank}, timeout_s)
            if reply is None:
                raise TimeoutError(f"no consumer on {host}:{self.port}")
            info = unpack(reply)
            from kvserve_hpdps_b200.parallel.p2p import PeerMapping
            self._peer = PeerMapping(local_rank, info["handle"], info["nbytes"])
            self.ring_bytes = int(info["ring_bytes"])
            self.flag_off = int(info["flag_off"])
            self.n_flags = int(info["n_flags"])
            self._alloc = RingAllocator(self.ring_bytes)
            self._stream = torch.cuda.Stream(device=self.device)
            self._seq = 0
            self._inflight_msgs = 0
            self._lock = threading.Lock()
            self._slots_cv = threading.Condition(self._lock)  # FREE returned flag slots
            self._free_slots: deque = deque(range(self.n_flags))
            self._slot_of: dict[int, int] = {}  # ring offset of a message -> its flag slot
            self._bw_lock = threading.Lock()
            self._bw_cache: Optional[tuple[float, float]] = None  # (MB/s, time measured)
            self._bw_probe = None  # (event, pinned stamps, ring offset, bytes, device stamps)
            self._probe_src: Optional[torch.Tensor] = None
            self._sent: dict[str, int] = defaultdict(int)
            self._failed: dict[str, int] = defaultdict(int)
            self._listeners: list = []
            # (done event, request_id, member_tids, nbytes, t0, ring offset)
            self._pending: deque = deque()
            self._aborted: list = []  # (event, ring offset, size) of uncommitted messages
            self._unfinished: set = set()  # ring offsets whose stores may still be landing
            self._free_after_done: dict = {}  # offset -> size, FREE seen before completion
            self._pending_cv = threading.Condition()
            self._io = threading.Thread(target=self._producer_io, daemon=True, name="kvs-p2p-io")
            self._io.start()
            self._done = threading.Thread(target=self._completion_loop, daemon=True,
                                          name="kvs-p2p-done")
            self._done.start()
        else:
            from kvserve_hpdps_b200.parallel.p2p import DeviceRegion
            self.n_flags = n_flags
            self.ring_bytes = int(ring_bytes)
            self.flag_off = _align(self.ring_bytes)
            self._region = DeviceRegion(local_rank, self.flag_off + n_flags * FLAG_STRIDE)
            self._ctl = ConsumerChannel(self.port)
            self._producer_id: Optional[bytes] = None
            self._lock = threading.Lock()
            self._arrived = threading.Condition(self._lock)
            self._received: dict[str, deque] = defaultdict(deque)
            self._releases: deque = deque()  # (event, off, size)
            self._io = threading.Thread(target=self._consumer_io, daemon=True, name="kvs-p2p-io")
            self._io.start()

    # ============================================================ producer
    def _producer_io(self) -> None:
        while not self._closed:
            try:
                while True:
                    try:
                        self._ctl.send(self._outbox.get_nowait())
                    except queue.Empty:
                        break
                raw = self._ctl.recv_or_wake(0.05)  # woken at once by a queued header
                if raw is None:
                    continue
                msg = unpack(raw)
                if msg.get("cmd") == "FREE":
                    self._on_free(msg["regions"])
            except Exception as e:  # noqa: BLE001
                if self._closed:  # the socket went away under close()
                    break
                logger.error("p2p producer io error: %s", e)

    def _send_ctl(self, msg: dict) -> None:
        """Queue a control message for the io thread (which owns the socket)
        and wake it, so the header leaves without waiting out its poll."""
        self._outbox.put(msg)
        self._ctl.wake()

    def _on_free(self, regions) -> None:
        """The consumer returned these (offset, size) ring regions.  A region
        whose message's own stores may still be landing (the consumer can
        refuse a header before the producer's kernels finished, and a raw
        or direct message's stores run on the producer's compute stream, not
        on the transfer stream) is released only once the completion thread
        has seen that message's done-event; the others go back at once, flag
        slot first (once its ring space is released, an offset can belong to
        a new message), then the space."""
        now = []
        with self._lock:
            for off, size in regions:
                off, size = int(off), int(size)
                if off in self._unfinished:
                    self._free_after_done[off] = size
                else:
                    now.append((off, size))
        self._release_regions(now)

    def _release_regions(self, regions) -> None:
        if not regions:
            return
        owned = []
        with self._lock:
            for off, size in regions:
                slot = self._slot_of.pop(int(off), None)
                if slot is None:  # not (or no longer) a message of ours
                    logger.error("p2p: FREE of unknown ring region at %d ignored", off)
                    continue
                self._free_slots.append(slot)
                owned.append((off, size))
            self._inflight_msgs -= len(owned)
            self._slots_cv.notify_all()
        for off, size in owned:
            self._alloc.release(off, size)

    def _completion_loop(self) -> None:
        while not self._closed:
            self._poll_probe()
            with self._pending_cv:
                while not self._pending and not self._aborted and not self._closed:
                    self._pending_cv.wait(timeout=0.2)
                    self._poll_probe()
                if self._closed:
                    return
                aborted = list(self._aborted)
                self._aborted.clear()
                item = self._pending[0] if self._pending else None
            self._release_aborted(aborted)
            if item is None:
                continue
            ev, rid, tids, nbytes, t0, base = item
            ev.synchronize()
            start = t0 if isinstance(t0, torch.cuda.Event) else None
            with self._pending_cv:
                self._pending.popleft()
                self._pending_cv.notify_all()
            with self._lock:  # a message without member ids counts for its request id
                for t in (tids or [rid]):
                    self._sent[t] += 1
            self._message_done(base)
            if isinstance(nbytes, tuple):  # (device count, host addend): coded stream size
                nbytes = int(nbytes[0].item()) + int(nbytes[1])
            # device time from the message's first kernel to its last store
            ms = start.elapsed_time(ev) if start is not None else (time.monotonic() - t0) * 1e3
            write_transfer_stats(rid, ms, nbytes, transport="nvlink-p2p")
            notify_sent(self._listeners, rid, list(tids or [rid]), ms, nbytes, logger)

    def _release_aborted(self, aborted) -> None:
        """Messages reserved but never committed: their ring space and flag
        slot go back once the work queued before the abort has finished."""
        for ev, off, size in aborted:
            if ev is not None:
                ev.synchronize()
            with self._lock:
                self._unfinished.discard(off)
                self._free_after_done.pop(off, None)
            self._release_regions([(off, size)])

    def _abandon(self, base: int, total: int, stream, request_id: str,
                 member_tids: Optional[list[str]], err: Exception) -> None:
        """A reserved message whose kernels could not be enqueued: it counts
        as failed and its region returns through the completion thread (after
        whatever ``stream`` had queued, which may still touch the region)."""
        try:
            done = stream.record_event()
        except Exception:  # noqa: BLE001 - the device may be what failed
            done = None
        with self._pending_cv:
            self._aborted.append((done, base, total))
            self._pending_cv.notify_all()
        self._unsent(request_id, member_tids, err)

    def _message_done(self, base: int) -> None:
        """The stores of the message at ring offset ``base`` have finished: a
        FREE that arrived before now releases its region and slot here."""
        with self._lock:
            self._unfinished.discard(base)
            late = self._free_after_done.pop(base, None)
        if late is not None:
            self._release_regions([(base, late)])

    def _track(self, done, request_id, member_tids, nbytes, t0, base) -> None:
        with self._pending_cv:
            self._pending.append((done, request_id, member_tids, nbytes, t0, base))
            self._pending_cv.notify_all()

    def _put(self, request_id: str, layer_names: list[str], tensors: list[torch.Tensor],
             n_body: int, meta: Optional[dict], kind: str,
             member_tids: Optional[list[str]]) -> None:
        sizes = [t.numel() * t.element_size() for t in tensors]
        offs, total = [], 0
        for s in sizes:
            offs.append(total)
            total += _align(s)
        trailer = total           # 16-byte message checksum after the payload
        total = total + ALIGN
        try:
            base, seq, slot = self._reserve(total)
        except RuntimeError as e:
            self._unsent(request_id, member_tids, e)
            return
        from kvserve_hpdps_b200.ops import kernels as K
        ready = _timing_event(torch.cuda.current_stream(self.device))
        try:
            with torch.cuda.stream(self._stream):
                self._stream.wait_event(ready)
                ck = torch.empty(2, dtype=torch.int64, device=self.device)
                K.zero_checksum(ck)
                # one pass: the copy over NVLink also sums the message checksum,
                # and its last CTA stores the checksum and publishes the flag
                segs = [(t.data_ptr(), self._peer.ptr + base + o, s, o)
                        for t, o, s in zip(tensors, offs, sizes)]
                K.copy_segments(segs, self.device, flag_ptr=self._peer.ptr + self.flag_off +
                                slot * FLAG_STRIDE, flag_value=seq & 0xFFFFFFFF, ck=ck,
                                trailer_ptr=self._peer.ptr + base + trailer)
                for t in tensors + [ck]:
                    t.record_stream(self._stream)
                done = _timing_event(self._stream)
        except Exception as e:  # noqa: BLE001
            self._abandon(base, total, self._stream, request_id, member_tids, e)
            return
        self._send_ctl({
            "cmd": "PUT_RING", "kind": kind, "request_id": request_id,
            "layer_names": list(layer_names), "meta": meta, "n_body": n_body,
            "specs": [{"shape": list(t.shape), "dtype": str(t.dtype).replace("torch.", ""),
                       "off": base + o, "nbytes": s} for t, o, s in zip(tensors, offs, sizes)],
            "region": [base, total], "slot": slot, "seq": seq, "trailer": base + trailer})
        self._track(done, request_id, member_tids, sum(sizes), ready, base)

    def _reserve(self, total: int) -> tuple[int, int, int]:
        """Ring space, sequence number and flag slot of a new message.

        A flag slot belongs to one message from here until the consumer's FREE
        of that message's ring region returns it (messages may be returned
        out of order), so a slot is never rewritten while its message is
        pending.  With every slot taken this waits at most ``timeout_s``."""
        deadline = time.monotonic() + self.timeout_s
        with self._slots_cv:
            if not self._free_slots:
                logger.warning("p2p: %d messages in flight, waiting for the consumer",
                               self._inflight_msgs)
            while not self._free_slots:
                left = deadline - time.monotonic()
                if left <= 0:
                    raise RuntimeError(f"{self._inflight_msgs} messages unreturned by the "
                                       f"consumer for {self.timeout_s}s")
                self._slots_cv.wait(timeout=min(left, 0.1))
            slot = self._free_slots.popleft()
            self._inflight_msgs += 1
        base = self._alloc.alloc(total, self.timeout_s)
        with self._slots_cv:
            if base is None:
                self._free_slots.appendleft(slot)
                self._inflight_msgs -= 1
                self._slots_cv.notify_all()
                raise RuntimeError(f"receive ring full for {self.timeout_s}s "
                                   f"({total} bytes needed)")
            self._seq += 1
            self._slot_of[base] = slot
            self._unfinished.add(base)
            return base, self._seq, slot

    def record_unsent(self, request_id: str, member_tids: Optional[list[str]],
                      err: Exception) -> None:
        """Count a message its producer could not send (e.g. no ring space)."""
        self._unsent(request_id, member_tids, err)

    def _unsent(self, request_id: str, member_tids: Optional[list[str]], err: Exception) -> None:
        """A message that got no ring space in time is dropped (logged) and
        counted in ``failed_layers``, as a refused message of the NCCL
        transport; the consumer's load times out for it."""
        logger.error("p2p: %s not sent: %s", request_id, err)
        with self._lock:
            for t in (member_tids or [request_id]):
                self._failed[t] += 1

    # ------------------------------------------------ direct-to-ring messages
    def open_message(self, sizes: list[int]) -> "RingMessage":
        """Reserve ring space for a message whose tensors (``sizes`` bytes
        each, in order) producer kernels will write straight into the
        consumer's ring.  Returns the device addresses to write, the message
        checksum accumulators (zeroed on the current stream) and the ready
        flag to publish; :meth:`commit_message` sends the header.  Raises
        RuntimeError when no ring space or flag slot frees up in time."""
        assert self.is_sender
        offs, total = [], 0
        for n in sizes:
            offs.append(total)
            total += _align(int(n))
        trailer = total
        total += ALIGN
        base, seq, slot = self._reserve(total)
        from kvserve_hpdps_b200.ops import kernels as K
        ck = torch.empty(2, dtype=torch.int64, device=self.device)
        K.zero_checksum(ck)
        ptr = self._peer.ptr + base
        return RingMessage(base=base, total=total, seq=seq, slot=slot, offsets=offs,
                           sizes=[int(n) for n in sizes], ptrs=[ptr + o for o in offs],
                           trailer_ptr=ptr + trailer, trailer_off=base + trailer, ck=ck,
                           flag_ptr=self._peer.ptr + self.flag_off + slot * FLAG_STRIDE,
                           flag_value=seq & 0xFFFFFFFF,
                           t0=_timing_event(torch.cuda.current_stream(self.device)))

    def view(self, msg: "RingMessage", i: int, dtype: torch.dtype = torch.uint8,
             shape=None) -> torch.Tensor:
        """Zero-copy tensor over tensor ``i`` of an open message (peer memory:
        only this framework's own kernels may write or read it)."""
        n = msg.sizes[i]
        esz = torch.empty((), dtype=dtype).element_size()
        return tensor_view(msg.ptrs[i], n, dtype, shape if shape is not None else [n // esz],
                           self.local_rank)

    def commit_message(self, msg: "RingMessage", request_id: str, layer_names: list[str],
                       meta: Optional[dict], specs: list[dict], n_body: int,
                       kind: str = "bundle", member_tids: Optional[list[str]] = None,
                       dyn_len: Optional[dict] = None,
                       sent_bytes: Optional[torch.Tensor] = None) -> None:
        """Send the header of a message whose kernels have been enqueued on
        the current stream (the last of them publishes ``msg.flag_value``).
        ``specs`` give each tensor's shape and dtype; ``dyn_len`` = {"seg":
        i, "len_off": o, "len_add": a} marks tensor i as a coded stream whose
        length (read on the device at byte o of the tensor, plus a) bounds
        the checksum; ``sent_bytes`` (int64 on the device) is the number of
        bytes that actually crossed the link, read by the completion thread
        for the transfer statistics."""
        done = _timing_event(torch.cuda.current_stream(self.device))
        full = []
        for sp, off, n in zip(specs, msg.offsets, msg.sizes):
            full.append({"shape": list(sp["shape"]), "dtype": sp["dtype"],
                         "off": msg.base + off, "nbytes": n})
        hdr = {"cmd": "PUT_RING", "kind": kind, "request_id": request_id,
               "layer_names": list(layer_names), "meta": meta, "n_body": n_body,
               "specs": full, "region": [msg.base, msg.total], "slot": msg.slot, "seq": msg.seq,
               "trailer": msg.trailer_off}
        if dyn_len is not None:
            hdr["dyn_len"] = dict(dyn_len)
        self._send_ctl(hdr)
        nbytes = sum(msg.sizes) if sent_bytes is None else sent_bytes
        self._track(done, request_id, member_tids, nbytes, msg.t0, msg.base)

    def abort_message(self, msg: "RingMessage", request_id: str,
                      member_tids: Optional[list[str]], err: Exception) -> None:
        """Give up a message after :meth:`open_message` (nothing was
        committed): its ring space and flag slot return once the work already
        queued on the current stream has finished, and it counts as failed."""
        done = torch.cuda.current_stream(self.device).record_event()
        with self._pending_cv:
            self._aborted.append((done, msg.base, msg.total))
        self._unsent(request_id, member_tids, err)

    def send_paged(self, request_id: str, layer_names: list[str], kv_layers: list[torch.Tensor],
                   block_ids, member_tids: Optional[list[str]] = None) -> None:
        """Raw (uncompressed) KV of one request straight from the paged
        caches into the consumer's ring: one gather launch over every layer,
        storing over NVLink, that also computes the message checksum and
        publishes the ready flag.  It runs on the current stream, so it is
        ordered before any later kernel that rewrites those blocks.  The
        consumer sees the stacked ``[L, 2, nb, bs, H, D]`` raw tensor."""
        assert self.is_sender
        from kvserve_hpdps_b200.ops import kernels as K
        ids = [int(b) for b in block_ids]
        raw = K.RawItems(kv_layers, [(l, ids) for l in range(len(kv_layers))])
        nbytes = raw.flat_bytes
        trailer = _align(nbytes)
        total = trailer + ALIGN
        try:
            base, seq, slot = self._reserve(total)
        except RuntimeError as e:
            self._unsent(request_id, member_tids, e)
            return
        dev = raw.device
        stream = torch.cuda.current_stream(dev)
        t0 = _timing_event(stream)
        try:
            ck = torch.empty(2, dtype=torch.int64, device=dev)
            K.paged_raw(raw, self._peer.ptr + base, True,
                        flag_ptr=self._peer.ptr + self.flag_off + slot * FLAG_STRIDE,
                        flag_value=seq & 0xFFFFFFFF, trailer_ptr=self._peer.ptr + base + trailer,
                        checksum=ck)
        except Exception as e:  # noqa: BLE001
            self._abandon(base, total, stream, request_id, member_tids, e)
            return
        done = _timing_event(stream)
        shape = [len(kv_layers), 2, len(ids)] + list(raw.block_shape)
        self._send_ctl({
            "cmd": "PUT_RING", "kind": "raw", "request_id": request_id,
            "layer_names": list(layer_names), "meta": None, "n_body": 1,
            "specs": [{"shape": shape, "dtype": str(raw.dtype).replace("torch.", ""),
                       "off": base, "nbytes": nbytes}],
            "block_order": raw.block_order,
            "region": [base, total], "slot": slot, "seq": seq, "trailer": base + trailer})
        self._track(done, request_id, member_tids, nbytes, t0, base)

    def bandwidth_mbps(self, probe_bytes: int = 64 << 20, max_age_s: float = 30.0,
                       timeout_s: float = 5.0, wait: bool = False) -> Optional[float]:
        """Device-timed push bandwidth to the consumer in MB/s (1 MB = 2^20
        bytes): ``probe_bytes`` are stored into a temporarily reserved part of
        the consumer's ring by the probe kernel, timed between the first CTA's
        start and the last CTA's end (globaltimer), with no host round trip in
        the measured interval.

        The caller never waits on the device (the controller calls this from
        the engine thread): the cached value is returned (None before the
        first measurement, when the caller falls back to its configured
        bandwidth), and a value older than ``max_age_s`` starts a new probe on
        the transfer stream.  The probe's stamps reach pinned host memory by a
        stream-ordered copy; the completion thread (or a later call) reads
        them once the probe's event has passed.  ``wait=True`` blocks until
        the probe finished, at most ``timeout_s`` (start-up and tests)."""
        assert self.is_sender
        self._poll_probe()
        now = time.monotonic()
        with self._bw_lock:
            cached = self._bw_cache
            if (cached is None or now - cached[1] >= max_age_s) and self._bw_probe is None:
                self._start_probe(int(probe_bytes))
            probe = self._bw_probe
        if wait and probe is not None:
            deadline = time.monotonic() + timeout_s
            while not probe[0].query() and time.monotonic() < deadline:
                time.sleep(0.001)
            self._poll_probe()
        cached = self._bw_cache
        return cached[0] if cached else None

    def _start_probe(self, probe_bytes: int) -> None:
        """Launch one probe (caller holds _bw_lock); skipped when the ring
        has no room right now."""
        from kvserve_hpdps_b200.ops import kernels as K
        n = _align(probe_bytes)
        with self._alloc.cv:
            base = self._alloc.try_alloc(n)
        if base is None:
            return
        with torch.cuda.device(self.device), torch.cuda.stream(self._stream):
            src = self._probe_src
            if src is None or src.numel() < n:
                src = torch.zeros(n, dtype=torch.uint8, device=self.device)
                self._probe_src = src
            stamps = torch.empty(2, dtype=torch.int64, device=self.device)
            stamps[0].fill_(2 ** 63 - 1)
            stamps[1].fill_(0)
            K.probe_push(src, self._peer.ptr + base, n, stamps)
            host = torch.empty(2, dtype=torch.int64, pin_memory=True)
            host.copy_(stamps, non_blocking=True)
            ev = self._stream.record_event()
        self._bw_probe = (ev, host, base, n, stamps)

    def _poll_probe(self) -> None:
        """Finish a probe whose event has passed (no device wait)."""
        with self._bw_lock:
            probe = self._bw_probe
            if probe is None or not probe[0].query():
                return
            self._bw_probe = None
        ev, host, base, n, _ = probe
        self._alloc.release(base, n)
        t0, t1 = (int(v) for v in host.tolist())
        if t1 > t0:
            self._bw_cache = (n / (1 << 20) / ((t1 - t0) * 1e-9), time.monotonic())

    def send(self, request_id: str, layer_names: list[str], stacked_kv: torch.Tensor) -> None:
        assert self.is_sender
        self._put(request_id, layer_names, [stacked_kv.to(self.device).contiguous()], 1, None,
                  "raw", None)

    def send_bundle(self, request_id: str, layer_names: list[str], meta: dict,
                    body_chunks: list[torch.Tensor], aux_tensors: list[torch.Tensor],
                    member_tids: Optional[list[str]] = None) -> None:
        assert self.is_sender
        body = [t.to(self.device).contiguous() for t in body_chunks]
        aux = [t.to(self.device).contiguous() for t in aux_tensors]
        self._put(request_id, layer_names, body + aux, len(body), meta, "bundle", member_tids)

    def sent_layers(self, transfer_id: str) -> int:
        with self._lock:
            return self._sent.get(transfer_id, 0)

    def add_sent_listener(self, fn) -> None:
        """``fn(request_id, transfer_ids, latency_ms)`` on the completion thread
        once a message's stores have finished (time from its send call); a
        listener that takes an ``nbytes`` keyword also gets the bytes that
        crossed the link (for a coded stream, its exact length)."""
        self._listeners.append(fn)

    def failed_layers(self, transfer_id: str) -> int:
        with self._lock:
            return self._failed.get(transfer_id, 0)

    def clear_sent(self, transfer_id: str) -> None:
        with self._lock:
            self._sent.pop(transfer_id, None)
            self._failed.pop(transfer_id, None)

    def wait_for_sent(self, timeout_s: Optional[float] = None) -> bool:
        deadline = None if timeout_s is None else time.monotonic() + timeout_s
        with self._pending_cv:
            while self._pending:
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    return False
                self._pending_cv.wait(timeout=0.2 if left is None else min(left, 0.2))
        return True

    # ============================================================ consumer
    def _consumer_io(self) -> None:
        while not self._closed:
            try:
                self._flush_releases()
                got = self._ctl.poll(5)
                if got is None:
                    continue
                ident, msg = got
                cmd = msg.get("cmd")
                if cmd == "RING_HELLO":
                    self._producer_id = ident
                    self._ctl.reply(ident, pack({
                        "handle": self._region.ipc_handle(), "nbytes": self._region.nbytes,
                        "ring_bytes": self.ring_bytes, "flag_off": self.flag_off,
                        "n_flags": self.n_flags}))
                elif cmd == "PUT_RING":
                    try:
                        self._on_put(msg)
                    except Exception as e:  # noqa: BLE001
                        logger.error("p2p: unusable PUT_RING for %r: %s", msg.get("request_id"), e)
                        self._reject_put(msg)
                else:
                    logger.warning("p2p: unknown control message %r", cmd)
            except Exception as e:  # noqa: BLE001
                if self._closed:  # the socket went away under close()
                    break
                logger.error("p2p consumer io error: %s", e)

    def _reject_put(self, msg: dict) -> None:
        """A header that cannot be turned into tensors: the request is
        reported failed at once (no wait for the load timeout) and its ring
        region goes back to the producer, which reuses it (and its flag slot)
        only after this message's own stores have finished."""
        rid = msg.get("request_id")
        if isinstance(rid, str):
            with self._lock:
                self._received[rid].append((FAILED_LAYER_NAMES, FAILED_PAYLOAD))
                self._arrived.notify_all()
        region = msg.get("region")
        if (isinstance(region, (list, tuple)) and len(region) == 2
                and all(isinstance(v, int) for v in region) and self._producer_id is not None):
            self._ctl.reply(self._producer_id, pack({"cmd": "FREE", "regions": [list(region)]}))

    def _check_put(self, msg: dict) -> None:
        """A header's offsets address this GPU's own ring: every tensor, the
        checksum trailer and the flag slot must lie inside the message's
        region and the region inside the ring, and every shape must match its
        byte count, before any view or kernel touches them (a corrupt or
        foreign header is refused instead of read or written out of bounds)."""
        def whole(v) -> bool:
            return isinstance(v, int) and not isinstance(v, bool) and v >= 0
        region = msg.get("region")
        if not (isinstance(region, (list, tuple)) and len(region) == 2
                and all(whole(v) for v in region)):
            raise ValueError(f"bad region {region!r}")
        lo, hi = int(region[0]), int(region[0]) + int(region[1])
        if hi > self.ring_bytes:
            raise ValueError(f"region [{lo}, {hi}) outside the {self.ring_bytes}-byte ring")
        if not (whole(msg.get("slot")) and msg["slot"] < self.n_flags and whole(msg.get("seq"))):
            raise ValueError("bad flag slot or sequence number")
        if msg.get("kind") not in ("raw", "bundle"):
            raise ValueError(f"unknown message kind {msg.get('kind')!r}")
        specs = msg.get("specs")
        if not isinstance(specs, list) or not specs:
            raise ValueError("no tensor specs")
        for sp in specs:
            off, n, shape = sp.get("off"), sp.get("nbytes"), sp.get("shape")
            if not (whole(off) and whole(n) and lo <= off and off + n <= hi):
                raise ValueError(f"tensor [{off}, +{n}) outside its region")
            dt = getattr(torch, sp["dtype"], None) if isinstance(sp.get("dtype"), str) else None
            if not isinstance(dt, torch.dtype) or not isinstance(shape, list) \
                    or not all(whole(d) for d in shape):
                raise ValueError(f"bad tensor spec {sp!r}")
            numel = 1
            for d in shape:
                numel *= d
            if numel * dt.itemsize != n:
                raise ValueError(f"shape {shape} of {sp['dtype']} is not {n} bytes")
        tr = msg.get("trailer")
        if tr is not None and not (whole(tr) and lo <= tr and tr + 16 <= hi):
            raise ValueError("checksum trailer outside its region")
        if msg["kind"] == "bundle" and not (whole(msg.get("n_body"))
                                            and msg["n_body"] <= len(specs)):
            raise ValueError("bad body count")

    def _on_put(self, msg: dict) -> None:
        self._check_put(msg)
        views = [tensor_view(self._region.ptr + s["off"], s["nbytes"], getattr(torch, s["dtype"]),
                             s["shape"], self.local_rank) for s in msg["specs"]]
        ring = {"slot": msg["slot"], "seq": msg["seq"], "region": tuple(msg["region"]),
                "trailer": msg.get("trailer"),
                "segs": [(s["off"] - msg["region"][0], s["nbytes"]) for s in msg["specs"]]}
        dyn = msg.get("dyn_len")
        if dyn is not None:  # a coded stream: its length is in its own header
            i = int(dyn["seg"])
            if not 0 <= i < len(msg["specs"]) or not 0 <= int(dyn["len_off"]) <= \
                    msg["specs"][i]["nbytes"] - 8:
                raise ValueError("dyn_len outside its tensor")
            ring["dyn"] = (i, int(dyn["len_off"]), int(dyn["len_add"]))
        if msg["kind"] == "raw":
            payload = {"__ring_raw__": True, "tensor": views[0], "__ring__": ring,
                       "block_order": msg.get("block_order", "nhd")}
        else:
            n = msg["n_body"]
            payload = {"__bundle__": True, "meta": msg["meta"], "body_chunks": views[:n],
                       "aux_tensors": views[n:], "__ring__": ring}
        with self._lock:
            self._received[msg["request_id"]].append((msg["layer_names"], payload))
            self._arrived.notify_all()

    def wait_received(self, timeout_s: float) -> bool:
        """Block until some message is waiting to be drained or ``timeout_s``
        passes; True when a message is waiting."""
        assert not self.is_sender
        with self._arrived:
            if not any(self._received.values()):
                self._arrived.wait(timeout=timeout_s)
            return any(self._received.values())

    def drain_received(self) -> dict[str, list[tuple[list[str], Any]]]:
        assert not self.is_sender
        with self._lock:
            out = {k: list(v) for k, v in self._received.items() if v}
            self._received.clear()
        return out

    def prepare(self, payload: Any, device: Optional[torch.device] = None) -> None:
        """Make the current stream wait (bounded, on the device) until the
        payload's bytes have landed, then verify the message checksum the
        producer stored behind the payload (a mismatch records ERR_CORRUPT in
        the device error word; no host wait)."""
        if not isinstance(payload, dict) or "__ring__" not in payload:
            return
        from kvserve_hpdps_b200.ops import kernels as K
        r = payload["__ring__"]
        dev = device or self.device
        K.wait_flag(self._region.ptr + self.flag_off + r["slot"] * FLAG_STRIDE,
                    r["seq"] & 0xFFFFFFFF, dev, timeout_s=self.flag_timeout_s)
        if r.get("trailer") is not None:  # corruption -> ERR_CORRUPT in the device error word
            base = r["region"][0]
            segs = [(self._region.ptr + base + o, o, n) for o, n in r["segs"]]
            if r.get("dyn") is not None:  # checksum over the stream's own length only
                i, lo, la = r["dyn"]
                segs[i] = segs[i] + (segs[i][0] + lo, la)
            K.verify_checksum(segs, self._region.ptr + r["trailer"], dev)

    def release(self, payload: Any, device: Optional[torch.device] = None) -> None:
        """Return the payload's ring space once the work queued so far on the
        current stream (its decode) has finished."""
        if not isinstance(payload, dict) or "__ring__" not in payload:
            return
        ev = torch.cuda.current_stream(device or self.device).record_event()
        off, size = payload["__ring__"]["region"]
        with self._lock:
            self._releases.append((ev, off, size))

    def _flush_releases(self) -> None:
        done = []
        with self._lock:
            while self._releases and self._releases[0][0].query():
                _, off, size = self._releases.popleft()
                done.append([off, size])
        if done and self._producer_id is not None:
            self._ctl.reply(self._producer_id, pack({"cmd": "FREE", "regions": done}))

    def close(self) -> None:
        self._closed = True
        io = getattr(self, "_io", None)
        if io is not None and io is not threading.current_thread():
            io.join(timeout=1.0)  # its polls return within a few ms
        try:
            self._ctl.close()
        except Exception:  # noqa: BLE001
            pass


def is_ring_raw(payload: Any) -> bool:
    return isinstance(payload, dict) and payload.get("__ring_raw__", False)


__all__ = ["P2PTransport", "RingAllocator", "tensor_view", "is_ring_raw", "FAILED_PAYLOAD",
           "FAILED_LAYER_NAMES"]
