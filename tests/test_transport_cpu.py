"""Transport protocol tests on CPU: two processes over gloo, the ZMQ legacy
transport, and failure paths injected on the host (no GPU involved)."""

import multiprocessing as mp
import socket
import time

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
    tr.send("t_raw", ["l0", "l1"], torch.arange(12, dtype=torch.float32).view(2, 6))
    tr.send_bundle("t_bundle", ["__compressed__", "l0"], {"k": 1},
                   [torch.arange(5, dtype=torch.uint8)], [torch.ones(2, 3)],
                   member_tids=["a", "b"])
    tr.send("t_fail", ["l0"], torch.zeros(13, 13))
    ok = tr.wait_for_sent(60)
    q.put({"ok": ok, "sent_a": tr.sent_layers("a"), "sent_b": tr.sent_layers("b"),
           "sent_x": tr.sent_layers("x")})
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
