"""Connector on GPUs: the fused default-mode path through the in-process
transport (1 GPU, both overlap modes) and the NVLink ring transport between
two processes on two GPUs (raw and compressed)."""

import multiprocessing as mp
import os
import socket
import time
from types import SimpleNamespace

import pytest
import torch

os.environ.setdefault("KVSERVE_TRANSPORT", "fake")

pytestmark = pytest.mark.gpu

L, H, D, BS = 4, 4, 128, 16


def vllm_config(producer, compression, port=25010, transport=None):
    mc = SimpleNamespace(get_num_kv_heads=lambda pc: H, get_head_size=lambda: D,
                         get_num_layers=lambda pc: L, model="/m/Qwen2.5-7B-Instruct",
                         hf_text_config=SimpleNamespace(num_hidden_layers=L), use_mla=False)
    extra = {"compression": compression}
    if transport:
        extra["transport"] = transport
    kv = SimpleNamespace(is_kv_producer=producer, kv_ip="127.0.0.1", kv_port=port,
                         kv_connector_extra_config=extra)
    return SimpleNamespace(kv_transfer_config=kv, cache_config=SimpleNamespace(block_size=BS),
                           model_config=mc, parallel_config=SimpleNamespace())


def _caches(nblocks, seed, device, fill=True):
    g = torch.Generator(device="cpu").manual_seed(seed)
    out = {}
    for l in range(L):
        t = torch.randn(2, nblocks, BS, H, D, generator=g) if fill else torch.zeros(2, nblocks, BS, H, D)
        out[f"model.layers.{l}.self_attn.attn"] = t.to(device=device, dtype=torch.bfloat16)
    return out


def _meta(reqs):
    from kvserve_hpdps_b200.connector.compressed_kv_connector import CompressedKVConnectorMetadata
    m = CompressedKVConnectorMetadata()
    for rid, tid, ntok, blocks in reqs:
        m.add_request(rid, tid, list(range(ntok)), blocks, BS)
    return m


def _cos(a, b):
    return float(torch.nn.functional.cosine_similarity(a.float().flatten(), b.float().flatten(), dim=0))


@pytest.mark.parametrize("compression", ["default", None])
@pytest.mark.parametrize("overlap", ["off", "stream"])
def test_fused_default_handoff_in_process(overlap, compression, monkeypatch):
    """Both overlap modes, compressed and raw: in stream mode every layer goes
    out from save_kv_layer (one grouped message per layer compressed, one
    message per layer and request raw), in off mode one message per request."""
    monkeypatch.setenv("KVSERVE_OVERLAP_MODE", overlap)
    from kvserve_hpdps_b200.connector.compressed_kv_connector import (CompressedKVConnector,
                                                                      KVConnectorRole)
    from kvserve_hpdps_b200.parallel.fake_transport import FakeTransportPair
    pair = FakeTransportPair()
    p = CompressedKVConnector(vllm_config(True, compression), KVConnectorRole.WORKER)
    c = CompressedKVConnector(vllm_config(False, compression), KVConnectorRole.WORKER)
    p.attach_transport(pair.producer())
    c.attach_transport(pair.consumer())
    pc, cc = _caches(24, 1, "cuda"), _caches(24, 2, "cuda", fill=False)
    p.register_kv_caches(pc)
    c.register_kv_caches(cc)
    reqs_p = [("a", "ta", 100, [3, 9, 1, 17, 5, 20, 11]), ("b", "tb", 40, [0, 6, 22])]
    reqs_c = [("da", "ta", 100, [4, 2, 8, 10, 12, 14, 16]), ("db", "tb", 40, [23, 1, 3])]
    p.bind_connector_metadata(_meta(reqs_p))
    for name in sorted(pc):
        p.save_kv_layer(name, pc[name], None)
    p.wait_for_save()
    torch.cuda.synchronize()
    c.bind_connector_metadata(_meta(reqs_c))
    c.start_load_kv(None)
    torch.cuda.synchronize()
    for (rp, _, n, bp), (rc, _, _, bcs) in zip(reqs_p, reqs_c):
        for name in pc:
            src = pc[name][:, bp].reshape(2, -1, H, D)[:, :n]
            dst = cc[name][:, bcs].reshape(2, -1, H, D)[:, :n]
            if compression is None:
                assert torch.equal(src, dst), (rp, name)
            else:
                assert _cos(src, dst) > 0.9, (rp, name)
    if overlap == "stream":
        assert pair.messages == (L if compression else 2 * L)
    else:
        assert pair.messages == 2


@pytest.mark.parametrize("blocks_outer", [False, True], ids=["fa_layout", "fi_layout"])
def test_controller_mode_paged_handoff(blocks_outer, tmp_path, monkeypatch):
    """Controller mode with a library of fused profiles: the producer sends
    through the paged kernels (no dense copy of the request), the message
    names its profile and the consumer decodes with that profile's manager.
    Both cache layouts ([2, blocks, ...] and [blocks, 2, ...])."""
    monkeypatch.setenv("KVSERVE_OVERLAP_MODE", "off")
    from kvserve_hpdps_b200.connector.compressed_kv_connector import (CompressedKVConnector,
                                                                      KVConnectorRole)
    from kvserve_hpdps_b200.offline.library_export import build_library, write_library
    from kvserve_hpdps_b200.offline.search_space import Candidate
    from kvserve_hpdps_b200.parallel.fake_transport import FakeTransportPair

    def spec(cfg):
        return {"enabled": True, "pipeline": ["transformer", "quantizer", "codec"],
                "quantizer_config": dict(cfg), "codec_config": {"codec_type": "rans"},
                "min_compress_size": 0}
    evals = [{"candidate": c.key(), "config": c.quantizer_config(), "accuracy": acc,
              "compression_ratio": cr, "harmonic_speed_mbps": 30000.0}
             for c, acc, cr in [(Candidate(0.0, 16, 16, 8, 6), 0.995, 3.5),
                                (Candidate(0.8, 12, 8, 6, 4), 0.97, 6.0)]]
    path = tmp_path / "lib.json"
    write_library(str(path), build_library(evals, "Qwen2.5-7B-Instruct", spec_builder=spec))
    ctl = {"mode": "controller", "library_path": str(path), "epsilon": 0.0,
           "service_config": {"bandwidth_mbps": 150.0, "slo_ms": 1e9,
                              "accuracy_requirement": 0.96, "t_model_ms": 0.0}}
    pair = FakeTransportPair()
    p = CompressedKVConnector(vllm_config(True, ctl), KVConnectorRole.WORKER)
    c = CompressedKVConnector(vllm_config(False, ctl), KVConnectorRole.WORKER)
    p.attach_transport(pair.producer())
    c.attach_transport(pair.consumer())
    pc, cc = _caches(24, 1, "cuda"), _caches(24, 2, "cuda", fill=False)
    if blocks_outer:  # same values, [blocks, 2, bs, H, D]
        pc = {n: t.transpose(0, 1).contiguous() for n, t in pc.items()}
        cc = {n: t.transpose(0, 1).contiguous() for n, t in cc.items()}
    p.register_kv_caches(pc)
    c.register_kv_caches(cc)
    bp, bc, n = [3, 9, 1, 17, 5, 20, 11], [4, 2, 8, 10, 12, 14, 16], 100
    p.bind_connector_metadata(_meta([("a", "ta", n, bp)]))
    for name in sorted(pc):
        p.save_kv_layer(name, pc[name], None)
    p.wait_for_save()
    torch.cuda.synchronize()
    c.bind_connector_metadata(_meta([("da", "ta", n, bc)]))
    c.start_load_kv(None)
    torch.cuda.synchronize()
    comp_p, comp_c = p._get_compressor(), c._get_compressor()
    assert comp_p.supports_paged() and pair.messages == 1
    assert len(comp_p._manager_cache) == 1 and len(comp_c._manager_cache) == 1
    for name in pc:
        for plane in (0, 1):
            src = (pc[name][bp, plane] if blocks_outer else pc[name][plane, bp]).reshape(-1, H, D)[:n]
            dst = (cc[name][bc, plane] if blocks_outer else cc[name][plane, bc]).reshape(-1, H, D)[:n]
            assert _cos(src, dst) > 0.85, (name, plane)


def test_stream_mode_loads_layer_by_layer(monkeypatch):
    """Stream mode on the consumer: start_load_kv returns without waiting for
    the whole request, and wait_for_layer_load(l) makes layer l's KV (of
    every request of the step, grouped messages included) ready while the
    producer has not yet sent the last layer."""
    monkeypatch.setenv("KVSERVE_OVERLAP_MODE", "stream")
    import kvserve_hpdps_b200.connector.compressed_kv_connector as mod
    monkeypatch.setattr(mod, "LOAD_TIMEOUT_S", 20.0)
    from kvserve_hpdps_b200.connector.compressed_kv_connector import (CompressedKVConnector,
                                                                      KVConnectorRole)
    from kvserve_hpdps_b200.parallel.fake_transport import FakeTransportPair
    pair = FakeTransportPair()
    p = CompressedKVConnector(vllm_config(True, "default"), KVConnectorRole.WORKER)
    c = CompressedKVConnector(vllm_config(False, "default"), KVConnectorRole.WORKER)
    p.attach_transport(pair.producer())
    c.attach_transport(pair.consumer())
    pc, cc = _caches(24, 1, "cuda"), _caches(24, 2, "cuda", fill=False)
    p.register_kv_caches(pc)
    c.register_kv_caches(cc)
    reqs_p = [("a", "ta", 100, [3, 9, 1, 17, 5, 20, 11]), ("b", "tb", 40, [0, 6, 22])]
    reqs_c = [("da", "ta", 100, [4, 2, 8, 10, 12, 14, 16]), ("db", "tb", 40, [23, 1, 3])]
    names = sorted(pc, key=mod.layer_index)
    p.bind_connector_metadata(_meta(reqs_p))
    for name in names[:-1]:  # the last layer is not computed yet
        p.save_kv_layer(name, pc[name], None)
    torch.cuda.synchronize()

    def check(name):
        for (_, _, n, bp), (_, _, _, bcs) in zip(reqs_p, reqs_c):
            src = pc[name][:, bp].reshape(2, -1, H, D)[:, :n]
            dst = cc[name][:, bcs].reshape(2, -1, H, D)[:, :n]
            assert _cos(src, dst) > 0.9, name

    c.bind_connector_metadata(_meta(reqs_c))
    t0 = time.monotonic()
    c.start_load_kv(None)
    c.wait_for_layer_load(names[0])
    assert time.monotonic() - t0 < 5.0  # no wait for the missing layer
    torch.cuda.current_stream().synchronize()
    check(names[0])
    assert all(int(cc[names[-1]][:, b].abs().sum()) == 0 for _, _, _, b in reqs_c)
    p.save_kv_layer(names[-1], pc[names[-1]], None)
    p.wait_for_save()
    for name in names[1:]:
        c.wait_for_layer_load(name)
    torch.cuda.current_stream().synchronize()
    for name in names:
        check(name)
    assert pair.messages == L  # one grouped message per layer for both requests


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _role(producer, port, compression, q):
    try:
        torch.cuda.set_device(0 if producer else 1)
        os.environ["KVSERVE_TRANSPORT"] = "p2p"
        os.environ["KVSERVE_RING_BYTES"] = str(256 << 20)
        from kvserve_hpdps_b200.connector.compressed_kv_connector import (CompressedKVConnector,
                                                                          KVConnectorRole)
        conn = CompressedKVConnector(vllm_config(producer, compression, port, "p2p"),
                                     KVConnectorRole.WORKER)
        dev = torch.device("cuda", torch.cuda.current_device())
        caches = _caches(16, 7, dev, fill=producer)
        conn.register_kv_caches(caches)
        blocks_p, blocks_c = [5, 1, 12, 7, 3], [2, 9, 0, 14, 6]
        if producer:
            conn.bind_connector_metadata(_meta([("r", "t", 70, blocks_p)]))
            for name in sorted(caches):
                conn.save_kv_layer(name, caches[name], None)
            conn.wait_for_save()
            conn._transport.wait_for_sent(30)
            torch.cuda.synchronize()
            time.sleep(0.5)  # the listener that writes the statistics runs on its thread
            # device-timed NVLink push bandwidth (feeds the controller)
            bw = conn._transport.bandwidth_mbps(probe_bytes=32 << 20, wait=True)
            if bw is None or not 1e4 < bw < 2e6:
                raise RuntimeError(f"implausible probe bandwidth {bw} MB/s")
            time.sleep(2.0)
            rows = []
            path = os.environ.get("KVSERVE_COMPRESSION_STATS_PATH")
            if path and os.path.exists(path):
                import json
                with open(path) as f:
                    rows = [json.loads(line) for line in f]
            q.put(("p", rows))
        else:
            conn.bind_connector_metadata(_meta([("d", "t", 70, blocks_c)]))
            conn.start_load_kv(None)
            torch.cuda.synchronize()
            from kvserve_hpdps_b200.ops import kernels as K
            err = K.read_device_error(dev)
            ref = _caches(16, 7, dev, fill=True)
            cos = min(_cos(ref[n][:, blocks_p].reshape(2, -1, H, D)[:, :70],
                           caches[n][:, blocks_c].reshape(2, -1, H, D)[:, :70]) for n in caches)
            exact = all(torch.equal(ref[n][:, blocks_p], caches[n][:, blocks_c]) for n in caches)
            q.put(("c", (err, cos, exact)))
        conn.shutdown()
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put(("err", traceback.format_exc()))


# default-mode quantizer with one byte per code and no entropy coder
U8 = {"enabled": True, "pipeline": ["quantizer", "codec"],
      "quantizer_config": {"model_name": "Qwen2.5-7B-Instruct", "hybrid_ratio": 0.8,
                           "high_key_max_value": 12, "high_value_max_value": 8,
                           "low_key_max_value": 6, "low_value_max_value": 4},
      "codec_config": {"codec_type": "none"}}


@pytest.mark.multigpu
@pytest.mark.parametrize("compression", [None, "default", U8], ids=["raw", "default", "u8"])
def test_p2p_ring_handoff_two_gpus(compression, tmp_path, monkeypatch):
    """The connector pair over the NVLink ring: raw blocks, the default mode
    (the rANS compaction kernel stores only the coded stream into the
    consumer's ring) and byte codes (the quantize kernel stores them into the
    ring).  The statistics record the bytes that crossed the link."""
    monkeypatch.setenv("KVSERVE_COMPRESSION_STATS_PATH", str(tmp_path / "comp.jsonl"))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    c = ctx.Process(target=_role, args=(False, port, compression, q))
    c.start()
    time.sleep(3.0)
    p = ctx.Process(target=_role, args=(True, port, compression, q))
    p.start()
    results = {}
    for _ in range(2):
        k, v = q.get(timeout=240)
        assert k != "err", v
        results[k] = v
    p.join(60)
    c.join(60)
    err, cos, exact = results["c"]
    assert err == 0
    assert cos > 0.9
    if compression is None:  # raw blocks: one gather into the peer ring, one scatter
        assert exact
        return
    rows = results["p"]
    assert len(rows) == 1
    ratio = rows[0]["original_bytes"] / rows[0]["compressed_bytes"]
    if compression == "default":  # the coded stream's own size, not the reserved worst case
        assert ratio > 5.0, rows
    else:  # one byte per code plus the fp16 metadata
        assert 1.5 < ratio < 2.0, rows  # 70 of the 80 block rows hold tokens
