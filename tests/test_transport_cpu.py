"""Transport protocol tests on CPU: two processes over gloo, the ZMQ legacy
transport, and failure paths injected on the host (no GPU involved)."""

import multiprocessing as mp
import socket
import time
from collections import defaultdict, deque

import pytest
import torch


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _consumer(port, q, fail_rid):
    import kvserve_hpdps_b200.parallel.nccl_transport as nt
    orig = nt.alloc_from_spec

    def flaky(spec, device):
        if spec.get("shape") == [13, 13]:
            raise RuntimeError("injected allocation failure")
        return orig(spec, device)

    nt.alloc_from_spec = flaky
    tr = nt.NcclTransport(False, "127.0.0.1", port, backend="gloo", timeout_s=20)
    got = {}
    deadline = time.time() + 60
    while time.time() < deadline and sum(len(v) for v in got.values()) < 3:
        for k, v in tr.drain_received().items():
            got.setdefault(k, []).extend(v)
        time.sleep(0.01)
    out = {}
    for k, msgs in got.items():
        lst = []
        for names, payload in msgs:
            if payload is None:
                lst.append((names, None))
            elif isinstance(payload, dict):
                lst.append((names, {"meta": payload["meta"],
                                    "body": [t.tolist() for t in payload["body_chunks"]],
                                    "aux": [t.tolist() for t in payload["aux_tensors"]]}))
            else:
                lst.append((names, payload.tolist()))
        out[k] = lst
    q.put(out)
    tr.close()


def _producer(port, q):
    from kvserve_hpdps_b200.parallel.nccl_transport import NcclTransport
    tr = NcclTransport(True, "127.0.0.1", port, backend="gloo", timeout_s=20)
    heard = []
    tr.add_sent_listener(lambda rid, tids, ms: heard.append((rid, tids, ms >= 0)))
    tr.send("t_raw", ["l0", "l1"], torch.arange(12, dtype=torch.float32).view(2, 6))
    tr.send_bundle("t_bundle", ["__compressed__", "l0"], {"k": 1},
                   [torch.arange(5, dtype=torch.uint8)], [torch.ones(2, 3)],
                   member_tids=["a", "b"])
    tr.send("t_fail", ["l0"], torch.zeros(13, 13))
    ok = tr.wait_for_sent(60)
    q.put({"ok": ok, "sent_a": tr.sent_layers("a"), "sent_b": tr.sent_layers("b"),
           "sent_x": tr.sent_layers("x"), "failed": tr.failed_layers("t_fail"),
           "sent_fail": tr.sent_layers("t_fail"), "heard": heard})
    time.sleep(0.5)
    tr.close()


def test_nccl_transport_protocol_over_gloo():
    ctx = mp.get_context("spawn")
    port = free_port()
    qc, qp = ctx.Queue(), ctx.Queue()
    c = ctx.Process(target=_consumer, args=(port, qc, "t_fail"))
    c.start()
    time.sleep(1.0)
    p = ctx.Process(target=_producer, args=(port, qp))
    p.start()
    got = qc.get(timeout=90)
    prod = qp.get(timeout=90)
    p.join(30)
    c.join(30)
    assert prod["ok"] and prod["sent_a"] == 1 and prod["sent_b"] == 1 and prod["sent_x"] == 0
    assert prod["failed"] == 1 and prod["sent_fail"] == 0  # the refusal is counted
    assert prod["heard"] == [("t_raw", ["t_raw"], True), ("t_bundle", ["a", "b"], True)]
    assert got["t_raw"][0][0] == ["l0", "l1"]
    assert got["t_raw"][0][1] == torch.arange(12, dtype=torch.float32).view(2, 6).tolist()
    names, b = got["t_bundle"][0]
    assert names == ["__compressed__", "l0"] and b["meta"] == {"k": 1}
    assert b["body"] == [[0, 1, 2, 3, 4]] and b["aux"] == [[[1.0] * 3] * 2]
    assert got["t_fail"] == [([], None)]  # refused: FAILED sentinel, no hang


def test_zmq_transport_roundtrip():
    from kvserve_hpdps_b200.parallel.zmq_transport import ZmqTransport
    port = free_port()
    cons = ZmqTransport(False, "127.0.0.1", port)
    prod = ZmqTransport(True, "127.0.0.1", port)
    x = torch.randn(3, 2, 4).to(torch.bfloat16)
    prod.send("r1", ["a"], x)
    deadline = time.time() + 10
    got = {}
    while time.time() < deadline and "r1" not in got:
        got.update(cons.drain_received())
        time.sleep(0.01)
    assert got["r1"][0] == ["a"] and torch.equal(got["r1"][1], x)
    prod.close()
    cons.close()


def test_control_request_times_out_without_consumer():
    from kvserve_hpdps_b200.parallel.control import ProducerChannel
    ch = ProducerChannel("127.0.0.1", free_port(), timeout_s=0.2)
    t0 = time.time()
    assert ch.request({"cmd": "PUT"}, timeout_s=0.2) is None
    assert time.time() - t0 < 5
    ch.close()


def _collect(tr, want, seconds=60):
    got = {}
    deadline = time.time() + seconds
    while time.time() < deadline and sum(len(v) for v in got.values()) < want:
        for k, v in tr.drain_received().items():
            got.setdefault(k, []).extend(v)
        time.sleep(0.01)
    return got


def _plain_consumer(port, q, want, slow_first=0.0):
    import kvserve_hpdps_b200.parallel.nccl_transport as nt
    if slow_first:
        orig = nt.alloc_from_spec
        state = {"n": 0}

        def late(spec, device):  # answers the first header only after the producer gave up
            state["n"] += 1
            if state["n"] == 1:
                time.sleep(slow_first)
                raise RuntimeError("injected late refusal")
            return orig(spec, device)
        nt.alloc_from_spec = late
    tr = nt.NcclTransport(False, "127.0.0.1", port, backend="gloo", timeout_s=20)
    got = _collect(tr, want)
    q.put({k: [(n, None if p is None else p.tolist()) for n, p in v] for k, v in got.items()})
    time.sleep(0.5)
    tr.close()


def _bad_header_producer(port, q):
    from kvserve_hpdps_b200.parallel.control import ACK_REFUSED
    from kvserve_hpdps_b200.parallel.nccl_transport import NcclTransport
    tr = NcclTransport(True, "127.0.0.1", port, backend="gloo", timeout_s=20)
    out = {}
    for name, msg in (("no_rid", {"cmd": "PUT"}),
                      ("bad_dtype", {"cmd": "PUT", "request_id": "bad_dtype",
                                     "layer_names": ["l0"], "shape": [2], "dtype": "nope"}),
                      ("unknown", {"cmd": "WHAT"})):
        t0 = time.time()
        out[name] = (tr._ctl.request(msg, 20) == ACK_REFUSED, time.time() - t0)
    t0 = time.time()
    tr._ctl.sock.send(b"\xc1\xc1")  # 0xc1 is not a msgpack type byte
    out["garbage"] = (tr._ctl.recv(20) == ACK_REFUSED, time.time() - t0)
    tr.send("ok", ["l0"], torch.arange(6, dtype=torch.float32))
    out["sent"] = tr.wait_for_sent(60) and tr.sent_layers("ok") == 1 and not tr.ctl_failed
    q.put(out)
    time.sleep(0.5)
    tr.close()


def test_bad_headers_are_refused_and_the_pair_keeps_working():
    ctx = mp.get_context("spawn")
    port = free_port()
    qc, qp = ctx.Queue(), ctx.Queue()
    c = ctx.Process(target=_plain_consumer, args=(port, qc, 2))
    c.start()
    time.sleep(1.0)
    p = ctx.Process(target=_bad_header_producer, args=(port, qp))
    p.start()
    prod = qp.get(timeout=120)
    got = qc.get(timeout=120)
    p.join(30)
    c.join(30)
    for name in ("no_rid", "bad_dtype", "unknown", "garbage"):
        refused, seconds = prod[name]
        assert refused and seconds < 5, (name, prod[name])  # answered, not timed out
    assert prod["sent"]
    assert got["bad_dtype"] == [([], None)]  # FAILED sentinel for the refused request
    assert got["ok"] == [(["l0"], [0.0, 1.0, 2.0, 3.0, 4.0, 5.0])]


def _impatient_producer(port, q):
    from kvserve_hpdps_b200.parallel.nccl_transport import NcclTransport
    tr = NcclTransport(True, "127.0.0.1", port, backend="gloo", timeout_s=1.5)
    tr.send("slow", ["l0"], torch.zeros(4))
    ok1 = tr.wait_for_sent(30)
    t0 = time.time()
    tr.send("after", ["l0"], torch.ones(4))
    ok2 = tr.wait_for_sent(30)
    second_s = time.time() - t0
    time.sleep(3.0)  # the late refusal arrives meanwhile
    q.put({"ok": ok1 and ok2, "ctl_failed": tr.ctl_failed, "second_s": second_s,
           "sent": tr.sent_layers("slow") + tr.sent_layers("after"),
           "failed": tr.failed_layers("slow") + tr.failed_layers("after"),
           "stale": tr._ctl.discard_pending()})
    tr.close()


def test_producer_refuses_sends_after_a_control_timeout():
    """A header answered after the producer's timeout leaves the message
    order unknown: the producer refuses later sends at once instead of
    pairing their tensors with receives it cannot account for."""
    ctx = mp.get_context("spawn")
    port = free_port()
    qc, qp = ctx.Queue(), ctx.Queue()
    c = ctx.Process(target=_plain_consumer, args=(port, qc, 1, 4.0))
    c.start()
    time.sleep(1.0)
    p = ctx.Process(target=_impatient_producer, args=(port, qp))
    p.start()
    prod = qp.get(timeout=120)
    got = qc.get(timeout=120)
    p.join(30)
    c.join(30)
    assert prod["ok"] and prod["ctl_failed"] and prod["failed"] == 2 and prod["sent"] == 0
    assert prod["second_s"] < 1.0 and prod["stale"] == 1
    assert got == {"slow": [([], None)]}  # the consumer refused it (late); nothing else came


def _slot_state(n_flags, ring_bytes, timeout_s):
    """The producer-side slot and ring bookkeeping of a P2PTransport, without
    a device or a peer."""
    import threading
    from collections import deque

    from kvserve_hpdps_b200.parallel.p2p_transport import P2PTransport, RingAllocator
    t = object.__new__(P2PTransport)
    t.n_flags, t.timeout_s = n_flags, timeout_s
    t._lock = threading.Lock()
    t._slots_cv = threading.Condition(t._lock)
    t._free_slots = deque(range(n_flags))
    t._slot_of, t._inflight_msgs, t._seq = {}, 0, 0
    t._unfinished, t._free_after_done = set(), {}
    t._alloc = RingAllocator(ring_bytes)
    return t


def _reserve_done(t, n):
    """Reserve a message and mark its stores finished (what the completion
    thread does once the message's done-event has passed)."""
    m = t._reserve(n)
    t._message_done(m[0])
    return m


def test_p2p_flag_slots_are_reused_only_after_their_message_is_returned():
    import threading
    t = _slot_state(3, 1024, 0.3)
    a, b, c = (_reserve_done(t, 256) for _ in range(3))
    assert [m[1] for m in (a, b, c)] == [1, 2, 3]
    assert sorted(m[2] for m in (a, b, c)) == [0, 1, 2] and t._inflight_msgs == 3
    with pytest.raises(RuntimeError):  # every slot pending: bounded wait, then an error
        t._reserve(256)
    # returned out of order: the next message takes exactly the freed slot
    # (seq 4 modulo 3 would be b's slot, still pending)
    t._on_free([[a[0], 256]])
    d = _reserve_done(t, 256)
    assert d[1] == 4 and d[2] == a[2] and d[0] == a[0] and t._slot_of[d[0]] == a[2]
    # ring space short: the slot taken for the message goes back
    t._on_free([[b[0], 256]])
    with pytest.raises(RuntimeError):
        t._reserve(512)
    assert b[2] in t._free_slots and t._inflight_msgs == 2
    # a FREE from the io thread wakes a waiting reservation
    t.timeout_s = 5.0
    _reserve_done(t, 256)
    timer = threading.Timer(0.2, t._on_free, args=([[c[0], 256]],))
    timer.start()
    t0 = time.time()
    e = _reserve_done(t, 256)
    timer.join()
    assert e[2] == c[2] and 0.1 < time.time() - t0 < 3
    assert t._alloc.free_bytes() == 256 and t._inflight_msgs == 3  # [768, 1024) never used


def test_p2p_region_freed_early_waits_for_its_own_stores():
    """A consumer may return a message's region (e.g. it refused the header)
    while the producer's kernels for that message are still storing into it
    (raw and direct messages run on the producer's compute stream).  The
    region and its flag slot must not go to a new message before the
    completion thread has seen that message's done-event."""
    t = _slot_state(1, 512, 0.2)
    a = t._reserve(256)          # stores still in flight
    t._on_free([[a[0], 256]])    # refused at once by the consumer
    assert t._free_slots == deque() and t._inflight_msgs == 1
    with pytest.raises(RuntimeError):  # the only slot is still that message's
        t._reserve(256)
    t._message_done(a[0])        # its done-event passed: now it is returned
    assert list(t._free_slots) == [a[2]] and t._inflight_msgs == 0
    b = t._reserve(256)
    assert b[0] == a[0] and b[2] == a[2]


def _stress_producer(port, q, threads, per_thread):
    import threading

    from kvserve_hpdps_b200.parallel.nccl_transport import NcclTransport
    tr = NcclTransport(True, "127.0.0.1", port, backend="gloo", timeout_s=20)

    def worker(k):
        for i in range(per_thread):
            rid = f"t{k}-{i}"
            if i % 2:
                tr.send(rid, ["l0"], torch.full((k + 1, i + 1), float(i), dtype=torch.float32))
            else:
                tr.send_bundle(rid, ["__compressed__", "l0"], {"k": k, "i": i},
                               [torch.full((i + 3,), k, dtype=torch.uint8)], [],
                               member_tids=[rid, f"m{k}-{i}"])
    ts = [threading.Thread(target=worker, args=(k,)) for k in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    ok = tr.wait_for_sent(120)
    counts = {f"t{k}-{i}": tr.sent_layers(f"t{k}-{i}") for k in range(threads)
              for i in range(per_thread)}
    q.put({"ok": ok, "counts": counts, "failed": sum(tr.failed_layers(r) for r in counts)})
    time.sleep(0.5)
    tr.close()


def _stress_consumer(port, q, want):
    from kvserve_hpdps_b200.parallel.nccl_transport import NcclTransport
    tr = NcclTransport(False, "127.0.0.1", port, backend="gloo", timeout_s=20)
    got = _collect(tr, want, seconds=120)
    out = {}
    for rid, msgs in got.items():
        out[rid] = [(n, p["meta"], [t.tolist() for t in p["body_chunks"]]) if isinstance(p, dict)
                    else (n, None, p.tolist()) for n, p in msgs]
    q.put(out)
    time.sleep(0.5)
    tr.close()


def test_transport_under_concurrent_senders():
    """Host-thread stress: four threads send 25 messages each (raw and
    bundles) through one producer; every message arrives once and intact,
    and the send counters match."""
    threads, per = 4, 25
    ctx = mp.get_context("spawn")
    port = free_port()
    qc, qp = ctx.Queue(), ctx.Queue()
    c = ctx.Process(target=_stress_consumer, args=(port, qc, threads * per))
    c.start()
    time.sleep(1.0)
    p = ctx.Process(target=_stress_producer, args=(port, qp, threads, per))
    p.start()
    prod = qp.get(timeout=240)
    got = qc.get(timeout=240)
    p.join(30)
    c.join(30)
    assert prod["ok"] and prod["failed"] == 0
    assert all(v == 1 for v in prod["counts"].values())
    assert len(got) == threads * per
    for k in range(threads):
        for i in range(per):
            (names, meta, body), = got[f"t{k}-{i}"]
            if i % 2:
                assert names == ["l0"] and body == [[float(i)] * (i + 1)] * (k + 1)
            else:
                assert meta == {"k": k, "i": i} and body == [[k] * (i + 3)]


def test_p2p_consumer_rejects_unusable_headers():
    """A PUT_RING header whose payload cannot be mapped (here: no device)
    reports the request failed at once and returns its ring region."""
    import threading
    from collections import defaultdict, deque

    from kvserve_hpdps_b200.parallel.control import unpack
    from kvserve_hpdps_b200.parallel.p2p_transport import P2PTransport

    class Ctl:
        def __init__(self):
            self.sent = []

        def reply(self, ident, payload):
            self.sent.append((ident, unpack(payload)))

    t = object.__new__(P2PTransport)
    t._lock = threading.Lock()
    t._arrived = threading.Condition(t._lock)
    t._received = defaultdict(deque)
    t._ctl, t._producer_id = Ctl(), b"prod"
    t._region = type("R", (), {"ptr": 4096})()
    t.local_rank, t.is_sender = 0, False
    t.ring_bytes, t.n_flags = 1 << 20, 16
    msg = {"cmd": "PUT_RING", "kind": "bundle", "request_id": "r9", "layer_names": ["a"],
           "meta": {}, "n_body": 1, "region": [512, 1024], "slot": 3, "seq": 7,
           "specs": [{"shape": [4], "dtype": "uint8", "off": 512, "nbytes": 4}]}
    with pytest.raises(Exception):
        t._on_put(msg)  # tensor views need a CUDA device
    t._reject_put(msg)
    assert t.drain_received() == {"r9": [([], None)]}
    assert t._ctl.sent == [(b"prod", {"cmd": "FREE", "regions": [[512, 1024]]})]
    t._reject_put({"cmd": "PUT_RING"})  # nothing to report or return
    assert t.drain_received() == {} and len(t._ctl.sent) == 1


class _FakeEvent:
    def __init__(self):
        self.done = False

    def query(self):
        return self.done

    def synchronize(self):  # the engine thread must never wait on the device
        raise AssertionError("bandwidth_mbps waited on the device")


def test_p2p_bandwidth_probe_never_blocks_the_caller():
    """The controller reads the link bandwidth on the engine thread: the
    transport answers from its cache while a probe is in flight and takes
    the probe's result (globaltimer stamps copied to pinned host memory)
    only once its event has passed, releasing the probe's ring space."""
    import threading

    from kvserve_hpdps_b200.parallel.p2p_transport import P2PTransport, RingAllocator
    t = object.__new__(P2PTransport)
    t.is_sender = True
    t._bw_lock = threading.Lock()
    t._alloc = RingAllocator(1 << 20)
    base = t._alloc.try_alloc(1 << 18)
    ev = _FakeEvent()
    stamps = torch.tensor([1_000_000, 1_000_000 + 262_144], dtype=torch.int64)  # 262.144 us
    t._bw_cache = (5000.0, time.monotonic() - 100.0)  # stale: a probe is already running
    t._bw_probe = (ev, stamps, base, 1 << 18, None)
    t0 = time.monotonic()
    assert t.bandwidth_mbps() == 5000.0  # the old value, at once
    assert time.monotonic() - t0 < 0.05 and t._bw_probe is not None
    ev.done = True
    bw = t.bandwidth_mbps()  # finished probe: 256 KiB in 262.144 us = 953.67 MB/s
    assert t._bw_probe is None and abs(bw - (1 << 18) / (1 << 20) / 262.144e-6) < 1e-6
    assert t._alloc.free_bytes() == 1 << 20  # the probe's ring space is back


def test_p2p_reservation_whose_launch_failed_is_returned():
    """A message reserved in the ring whose kernels could not be enqueued
    counts as failed, and its region and flag slot go back after the work
    queued before the failure (the completion thread's job)."""
    import threading
    t = _slot_state(1, 512, 0.2)
    t._pending_cv = threading.Condition()
    t._aborted, t._failed = [], defaultdict(int)
    waited = []

    class Ev:
        def synchronize(self):
            waited.append(True)

    class Stream:
        def record_event(self):
            return Ev()

    base, seq, slot = t._reserve(256)
    t._abandon(base, 256 + 0, Stream(), "r", ["a", "b"], RuntimeError("launch failed"))
    assert t._failed == {"a": 1, "b": 1} and len(t._aborted) == 1
    with pytest.raises(RuntimeError):  # the only slot is still taken
        t._reserve(256)
    t._release_aborted(t._aborted)
    assert waited == [True] and list(t._free_slots) == [slot] and t._inflight_msgs == 0
    assert t._reserve(256)[0] == base


def test_p2p_consumer_checks_header_offsets_before_any_access():
    """Offsets in a PUT_RING header address the consumer's own ring: a
    header whose tensors, trailer, region or flag slot fall outside, or
    whose shape does not match its byte count, is refused before a view or
    kernel would touch the memory."""
    from kvserve_hpdps_b200.parallel.p2p_transport import P2PTransport
    t = object.__new__(P2PTransport)
    t.ring_bytes, t.n_flags = 4096, 8
    good = {"kind": "bundle", "n_body": 1, "region": [1024, 1024], "slot": 3, "seq": 9,
            "trailer": 1792, "specs": [{"shape": [256], "dtype": "uint8", "off": 1024,
                                         "nbytes": 256},
                                        {"shape": [2, 8], "dtype": "bfloat16", "off": 1280,
                                         "nbytes": 32}]}
    t._check_put(good)
    raw = dict(good, kind="raw", n_body=None)
    t._check_put(raw)

    def bad(**kw):
        m = dict(good)
        m.update(kw)
        with pytest.raises(ValueError):
            t._check_put(m)
    bad(region=[3584, 1024])                       # past the ring
    bad(region=[-256, 1024])
    bad(region=[1024])
    bad(slot=8)                                    # no such flag slot
    bad(slot=True)
    bad(kind="tensor")
    bad(trailer=2040)                              # trailer runs past the region
    bad(n_body=3)
    bad(specs=[])
    bad(specs=[{"shape": [256], "dtype": "uint8", "off": 900, "nbytes": 256}])   # before
    bad(specs=[{"shape": [1024], "dtype": "uint8", "off": 1280, "nbytes": 1024}])  # after
    bad(specs=[{"shape": [100], "dtype": "uint8", "off": 1024, "nbytes": 256}])  # shape
    bad(specs=[{"shape": [256], "dtype": "object", "off": 1024, "nbytes": 256}])
    bad(specs=[{"shape": [256], "dtype": "manual_seed", "off": 1024, "nbytes": 256}])
    t._check_put(dict(good, specs=[{"shape": [8], "dtype": "bool", "off": 1024, "nbytes": 8}]))
    bad(specs=[{"shape": [-1], "dtype": "uint8", "off": 1024, "nbytes": 0}])


def test_p2p_producer_headers_pass_the_consumer_check(monkeypatch):
    """Every header the producer builds (raw and bundle sends, paged raw
    sends, direct-to-ring messages) passes the consumer's offset check after
    the msgpack round trip: the kernels and CUDA events are stood in for on
    the CPU, the header dicts are the producer's own."""
    import threading
    from types import SimpleNamespace

    import kvserve_hpdps_b200.parallel.p2p_transport as PT
    from kvserve_hpdps_b200.ops import kernels as K
    from kvserve_hpdps_b200.parallel.control import pack, unpack

    class Stream:
        def wait_event(self, ev):
            pass

        def record_event(self):
            return None

    monkeypatch.setattr(PT, "_timing_event", lambda stream: None)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: Stream())
    monkeypatch.setattr(torch.cuda, "stream", lambda s: __import__("contextlib").nullcontext())
    monkeypatch.setattr(torch.Tensor, "record_stream", lambda self, s: None)
    for name in ("zero_checksum", "copy_segments", "paged_raw"):
        monkeypatch.setattr(K, name, lambda *a, **k: None)

    class Raw:  # the paged raw message's descriptors (device-built in production)
        def __init__(self, layers, items):
            self.flat_bytes = len(layers) * 2 * len(items[0][1]) * 16 * 4 * 128 * 2
            self.device, self.block_shape = torch.device("cpu"), (16, 4, 128)
            self.dtype, self.block_order = torch.bfloat16, "hnd"
    monkeypatch.setattr(K, "RawItems", Raw)

    ring, flags = 1 << 22, 8
    prod = _slot_state(flags, ring, 1.0)
    headers = []
    prod._send_ctl = headers.append
    prod._stream, prod.device, prod.local_rank = Stream(), torch.device("cpu"), 0
    prod.is_sender = True
    prod._peer = SimpleNamespace(ptr=1 << 40)
    prod.flag_off = ring
    prod._pending_cv, prod._pending = threading.Condition(), deque()
    prod._sent, prod._failed = defaultdict(int), defaultdict(int)
    cons = object.__new__(PT.P2PTransport)
    cons.ring_bytes, cons.n_flags = ring, flags

    prod.send("r0", ["l0"], torch.zeros(3, 2, 5, dtype=torch.bfloat16))
    prod.send_bundle("r1", ["__compressed__", "l0"], {"k": 1},
                     [torch.zeros(1000, dtype=torch.uint8)],
                     [torch.zeros(4, 128, dtype=torch.float16), torch.arange(3),
                      torch.zeros(0, dtype=torch.float32), torch.ones(5, dtype=torch.bool)])
    prod.send_paged("r2", ["l0", "l1"], [None, None], [4, 9, 1])
    msg = prod.open_message([16 + 70000, 1056])
    prod.commit_message(msg, "r3", ["__compressed__", "l0"], {"m": 2},
                        [{"shape": [16 + 70000], "dtype": "uint8"},
                         {"shape": [1056], "dtype": "uint8"}], 1,
                        dyn_len={"seg": 0, "len_off": 8, "len_add": 0})
    assert [h["request_id"] for h in headers] == ["r0", "r1", "r2", "r3"]
    for h in headers:
        cons._check_put(unpack(pack(h)))


def test_p2p_region_returned_twice_is_ignored():
    """A FREE repeated for the same region (or naming a region the producer
    never reserved) changes nothing: the free list never hands the same
    bytes to two messages and the in-flight count stays right."""
    from kvserve_hpdps_b200.parallel.p2p_transport import RingAllocator
    t = _slot_state(4, 2048, 0.2)
    a = _reserve_done(t, 512)
    b = _reserve_done(t, 512)
    t._on_free([[a[0], 512]])
    t._on_free([[a[0], 512]])          # repeated
    t._on_free([[1536, 512]])          # never reserved
    assert t._inflight_msgs == 1 and t._alloc.free_bytes() == 2048 - 512
    c = _reserve_done(t, 512)
    d = _reserve_done(t, 512)
    assert len({c[0], d[0], b[0]}) == 3  # three live messages, three regions
    al = RingAllocator(1024)
    off = al.try_alloc(256)
    assert al.release(off, 256) and not al.release(off, 256) and not al.release(900, 256)
    assert al.free_bytes() == 1024
