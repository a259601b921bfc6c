"""Connector tests on CPU with mocked vLLM objects and the in-process
transport: scheduler bookkeeping, producer -> consumer handoff (raw and
compressed through the generic pipeline) into different block ids, and
failure paths injected on the host."""

import os
from types import SimpleNamespace

import pytest
import torch

os.environ["KVSERVE_TRANSPORT"] = "fake"

from kvserve_hpdps_b200.connector.compressed_kv_connector import (  # noqa: E402
    CompressedKVConnector, CompressedKVConnectorMetadata, KVConnectorRole, layer_index)
from kvserve_hpdps_b200.parallel.fake_transport import FakeTransportPair  # noqa: E402

L, H, D, BS = 3, 4, 128, 16


def vllm_config(producer: bool, compression=None):
    mc = SimpleNamespace(get_num_kv_heads=lambda pc: H, get_head_size=lambda: D,
                         get_num_layers=lambda pc: L, model="/models/Qwen2.5-7B-Instruct",
                         hf_text_config=SimpleNamespace(num_hidden_layers=L), use_mla=False)
    kv = SimpleNamespace(is_kv_producer=producer, kv_ip="127.0.0.1", kv_port=25010,
                         kv_connector_extra_config={"compression": compression})
    return SimpleNamespace(kv_transfer_config=kv, cache_config=SimpleNamespace(block_size=BS),
                           model_config=mc, parallel_config=SimpleNamespace())


def make_pair(compression=None):
    pair = FakeTransportPair()
    p = CompressedKVConnector(vllm_config(True, compression), KVConnectorRole.WORKER)
    c = CompressedKVConnector(vllm_config(False, compression), KVConnectorRole.WORKER)
    p.attach_transport(pair.producer())
    c.attach_transport(pair.consumer())
    return p, c, pair


def caches(nblocks, seed):
    g = torch.Generator().manual_seed(seed)
    return {f"model.layers.{l}.self_attn.attn":
            torch.randn(2, nblocks, BS, H, D, generator=g).to(torch.bfloat16) for l in range(L)}


def meta_for(rid, tid, ntok, blocks):
    m = CompressedKVConnectorMetadata()
    m.add_request(rid, tid, list(range(ntok)), blocks, BS)
    return m


def handoff(p, c, ntok=40, src_blocks=(5, 1, 7), dst_blocks=(2, 6, 0)):
    pc, cc = caches(8, 1), caches(8, 2)
    p.register_kv_caches(pc)
    c.register_kv_caches(cc)
    p.bind_connector_metadata(meta_for("r1", "tid-1", ntok, list(src_blocks)))
    for name in sorted(pc, key=layer_index):
        p.save_kv_layer(name, pc[name], None)
    p.wait_for_save()
    c.bind_connector_metadata(meta_for("d1", "tid-1", ntok, list(dst_blocks)))
    c.start_load_kv(None)
    return pc, cc


def test_layer_index_and_layout():
    assert layer_index("model.layers.10.self_attn.attn") == 10
    assert CompressedKVConnector.get_required_kvcache_layout(vllm_config(True)) == "NHD"


def test_raw_handoff_is_exact():
    p, c, pair = make_pair(None)
    pc, cc = handoff(p, c)
    for name in pc:
        assert torch.equal(cc[name][:, [2, 6, 0]], pc[name][:, [5, 1, 7]])
    assert pair.messages == 1


def test_generic_compressed_handoff():
    spec = {"enabled": True, "pipeline": ["transformer", "quantizer", "codec"],
            "transformer_config": {"seed": 0x3333},
            "quantizer_config": {"hybrid_ratio": 0.3, "high_key_max_value": 16,
                                 "high_value_max_value": 16, "low_key_max_value": 12,
                                 "low_value_max_value": 12, "axis_key": "token",
                                 "axis_value": "token"},
            "codec_config": {"codec_type": "rans"}, "backend": "generic"}
    p, c, pair = make_pair(spec)
    pc, cc = handoff(p, c)
    for name in pc:
        a = pc[name][:, [5, 1, 7]].float().flatten()
        b = cc[name][:, [2, 6, 0]].float().flatten()
        assert float(torch.nn.functional.cosine_similarity(a, b, dim=0)) > 0.97
    # vLLM's connector-stats hooks: one message out, one request decoded
    ps, cs = p.get_kv_connector_stats(), c.get_kv_connector_stats()
    red = ps.reduce()
    assert red["Num messages sent"] == 1 and red["Compression ratio"] > 2.0
    assert ps.data["original_bytes"] == [L * 2 * 3 * BS * H * D * 2]
    assert cs.reduce()["Num decoded"] == 1 and cs.reduce()["Num failed loads"] == 0
    assert p.get_kv_connector_stats() is None  # the interval starts over


def test_connector_stats_aggregate_pickle_and_prometheus():
    import pickle

    from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram

    from kvserve_hpdps_b200.connector.metrics import KVServeConnectorStats
    a = KVServeConnectorStats()
    a.record_sent(1000, 250, 1.5, 2.0)
    a.record_decode(0.5)
    b = CompressedKVConnector.build_kv_connector_stats(pickle.loads(pickle.dumps(a)).data)
    b.record_sent(3000, 250, 0.5, 6.0)
    b.record_failed_load(2)
    agg = a.clone_and_reset().aggregate(b)
    assert a.is_empty() and not agg.is_empty()
    r = agg.reduce()
    assert r["Num messages sent"] == 3 and r["Compression ratio"] == round(5000 / 750, 3)
    assert r["Avg transfer time (ms)"] == round(10 / 3, 3) and r["Num failed loads"] == 2
    reg = CollectorRegistry()

    def bound(cls):
        return type(cls.__name__, (cls,), {"__init__": lambda self, *x, **k: cls.__init__(
            self, *x, registry=reg, **k)})
    types_ = {Gauge: bound(Gauge), Counter: bound(Counter), Histogram: bound(Histogram)}
    prom = CompressedKVConnector.build_prom_metrics(SimpleNamespace(kv_transfer_config=None),
                                                    types_, ["model", "engine"],
                                                    {0: ["m", "0"]})
    prom.observe(agg.data, 0)
    labels = {"model": "m", "engine": "0"}
    assert reg.get_sample_value("vllm:kvserve_wire_bytes_total", labels) == 750
    assert reg.get_sample_value("vllm:kvserve_original_bytes_total", labels) == 5000
    assert reg.get_sample_value("vllm:kvserve_transfer_seconds_count", labels) == 3
    assert reg.get_sample_value("vllm:kvserve_failed_loads_total", labels) == 2


def test_async_send_reports_raw_requests_finished():
    """With asynchronous sends the producer frees a request's blocks only
    after its message left; a raw (uncompressed) message counts too."""
    p, c, pair = make_pair(None)
    p._async_send = True
    handoff(p, c)
    done, _ = p.get_finished({"r1"})
    assert done == {"r1"}
    assert p.get_finished(set()) == (None, None)


def test_refused_and_dropped_messages_do_not_hang(monkeypatch):
    import kvserve_hpdps_b200.connector.compressed_kv_connector as mod
    monkeypatch.setattr(mod, "LOAD_TIMEOUT_S", 0.3)
    p, c, pair = make_pair(None)
    pair.refuse_next = 1
    pc, cc = handoff(p, c)  # FAILED sentinel: logged, blocks untouched
    assert not torch.equal(cc[next(iter(cc))][:, [2, 6, 0]], pc[next(iter(pc))][:, [5, 1, 7]])
    # the blocks go to vLLM's load-failure policy, once
    assert c.get_block_ids_with_load_errors() == {2, 6, 0}
    assert c.get_block_ids_with_load_errors() == set()
    assert c.get_kv_connector_stats().reduce()["Num failed loads"] == 1
    pair.drop_next = 1
    p2, c2, _ = p, c, pair
    handoff(p2, c2, dst_blocks=(3, 4, 5))  # nothing arrives: returns after the timeout
    assert c.get_block_ids_with_load_errors() == {3, 4, 5}
    handoff(p, c)  # a good handoff reports nothing
    assert c.get_block_ids_with_load_errors() == set()


def test_scheduler_side_bookkeeping():
    prod = CompressedKVConnector(vllm_config(True), KVConnectorRole.SCHEDULER)
    cons = CompressedKVConnector(vllm_config(False), KVConnectorRole.SCHEDULER)
    req = SimpleNamespace(request_id="r", prompt_token_ids=list(range(50)),
                          kv_transfer_params={"transfer_id": "T9"},
                          all_token_ids=list(range(51)))
    assert prod.get_num_new_matched_tokens(req, 0) == (0, False)
    assert cons.get_num_new_matched_tokens(req, 0) == (49, False)
    assert cons.get_num_new_matched_tokens(req, 49) == (0, False)
    blocks = SimpleNamespace(get_block_ids=lambda: ([3, 4, 5, 6],))
    cons.update_state_after_alloc(req, blocks, 49)
    prod.update_state_after_alloc(req, blocks, 0)
    new = SimpleNamespace(req_id="r", prompt_token_ids=list(range(50)), block_ids=([3, 4, 5, 6],),
                          num_computed_tokens=0)
    empty_cached = SimpleNamespace(req_ids=[], num_computed_tokens=[], new_block_ids=[],
                                   resumed_req_ids=set())
    so = SimpleNamespace(scheduled_new_reqs=[new], num_scheduled_tokens={"r": 50},
                         scheduled_cached_reqs=empty_cached)
    mc = cons.build_connector_meta(so)
    assert [(m.request_id, m.transfer_id, m.block_ids) for m in mc.requests] == [("r", "T9", [3, 4, 5, 6])]
    assert cons.build_connector_meta(so).requests == []  # loaded once
    mp = prod.build_connector_meta(so)
    assert mp.requests[0].transfer_id == "T9" and len(mp.requests[0].token_ids) == 50
    assert mp.requests[0].slot_mapping[:3].tolist() == [48, 49, 50]
    # chunked prefill: deferred until the whole prompt has KV
    so1 = SimpleNamespace(scheduled_new_reqs=[SimpleNamespace(
        req_id="c", prompt_token_ids=list(range(40)), block_ids=([1, 2],), num_computed_tokens=0)],
        num_scheduled_tokens={"c": 32}, scheduled_cached_reqs=empty_cached)
    assert prod.build_connector_meta(so1).requests == []
    cached = SimpleNamespace(req_ids=["c"], num_computed_tokens=[32], new_block_ids=[([9],)],
                             resumed_req_ids=set())
    so2 = SimpleNamespace(scheduled_new_reqs=[], num_scheduled_tokens={"c": 8},
                          scheduled_cached_reqs=cached)
    m2 = prod.build_connector_meta(so2)
    assert m2.requests[0].block_ids == [1, 2, 9]
    assert prod.request_finished(req, []) == (False, None)


def test_stats_files_and_summary(tmp_path, monkeypatch, capsys):
    """A compressed handoff writes one compression and one decode row; the
    summary joins them with transfer rows (a truncated row is skipped) into
    the mean compression ratio and the median compress + comm + decompress
    path."""
    import json

    from kvserve_hpdps_b200.utils import stats
    paths = {k: str(tmp_path / f"{k}.jsonl") for k in ("compression", "decode", "transfer")}
    monkeypatch.setenv("KVSERVE_COMPRESSION_STATS_PATH", paths["compression"])
    monkeypatch.setenv("KVSERVE_DECODE_STATS_PATH", paths["decode"])
    monkeypatch.setenv("KVSERVE_TRANSFER_STATS_PATH", paths["transfer"])
    spec = {"enabled": True, "pipeline": ["transformer", "quantizer", "codec"],
            "quantizer_config": {"hybrid_ratio": 0.3, "axis_key": "token",
                                 "axis_value": "token"},
            "codec_config": {"codec_type": "rans"}, "backend": "generic"}
    p, c, _ = make_pair(spec)
    handoff(p, c)
    crow = stats.read_rows(paths["compression"])
    assert len(crow) == 1 and len(stats.read_rows(paths["decode"])) == 1
    assert crow[0]["original_bytes"] == L * 2 * 3 * BS * H * D * 2
    stats.write_transfer_stats("r1", 2.0, 3_000_000, transport="fake")
    stats.write_transfer_stats("r2", 4.0, 5_000_000, transport="fake")
    with open(paths["transfer"], "a") as f:
        f.write('{"request_id": "r3", "transfer_ms": \n')
    s = stats.summarize(**paths)
    ratio = crow[0]["original_bytes"] / crow[0]["compressed_bytes"]
    assert s["avg_compression_ratio"] == pytest.approx(ratio) and ratio > 2
    assert s["transfer_rows"] == 2 and s["comm_ms"] == 3.0 and s["comm_mb"] == 4.0
    assert s["transports"] == ["fake"]
    assert s["xfer_path_ms"] == pytest.approx(s["compress_ms"] + 3.0 + s["decompress_ms"])
    assert s["xfer_if_overlap_ms"] == pytest.approx(s["compress_ms"] + 3.0)
    assert stats.main([]) == 0  # paths from the environment
    assert json.loads(capsys.readouterr().out)["transfer_rows"] == 2
    empty = stats.summarize(str(tmp_path / "missing.jsonl"))
    assert empty["avg_compression_ratio"] is None and empty["xfer_path_ms"] == 0.0


def test_load_timeout_bounds_the_whole_step(monkeypatch):
    """Three requests whose KV never arrives: the consumer's step returns
    after one load timeout, not one per request."""
    import time

    import kvserve_hpdps_b200.connector.compressed_kv_connector as mod
    monkeypatch.setattr(mod, "LOAD_TIMEOUT_S", 0.4)
    _, c, _ = make_pair(None)
    c.register_kv_caches(caches(8, 2))
    m = CompressedKVConnectorMetadata()
    for i in range(3):
        m.add_request(f"d{i}", f"missing-{i}", list(range(16)), [i], BS)
    c.bind_connector_metadata(m)
    t0 = time.monotonic()
    c.start_load_kv(None)
    assert 0.35 < time.monotonic() - t0 < 1.0
    assert c.get_block_ids_with_load_errors() == {0, 1, 2}


def test_async_send_frees_blocks_of_refused_requests():
    """A message the consumer refused still leaves the producer: with
    asynchronous sends the request is reported finished (its blocks are
    freed) instead of waiting for a send count that never comes."""
    p, c, pair = make_pair(None)
    p._async_send = True
    pair.refuse_next = 1
    handoff(p, c)
    assert p._transport.sent_layers("tid-1") == 0 and p._transport.failed_layers("tid-1") == 1
    done, _ = p.get_finished({"r1"})
    assert done == {"r1"} and p._transport.failed_layers("tid-1") == 0


def test_stream_mode_consumer_takes_raw_per_layer_messages():
    """The stream mode's fallback when compression fails: one raw message per
    layer and request ([1, 2, blocks, block_size, heads, dim]); the consumer
    waits for one message per layer and scatters each into its layer."""
    from kvserve_hpdps_b200.utils.kv_utils import extract_kv_from_layer_by_blocks
    p, c, pair = make_pair(None)
    c._overlap_mode, c._num_layers = "stream", L
    pc, cc = caches(8, 1), caches(8, 2)
    c.register_kv_caches(cc)
    for name in sorted(pc, key=layer_index):
        raw = extract_kv_from_layer_by_blocks(pc[name], [5, 1, 7]).unsqueeze(0)
        p._transport.send("tid-s", [name], raw)
    c.bind_connector_metadata(meta_for("d1", "tid-s", 40, [2, 6, 0]))
    c.start_load_kv(None)
    for name in pc:
        assert torch.equal(cc[name][:, [2, 6, 0]], pc[name][:, [5, 1, 7]])
    assert pair.messages == L


def test_controller_learns_from_compress_plus_transfer_time(tmp_path):
    """Controller mode: the latency fed to the bandit is the compression time
    plus the transfer time the transport reports once the message has left
    (here a 50 ms delivery delay), applied on the engine thread at the next
    step rather than right after the asynchronous send call."""
    import time

    from kvserve_hpdps_b200.offline.library_export import build_library, write_library
    from kvserve_hpdps_b200.offline.search_space import Candidate

    def spec(cfg):
        return {"enabled": True, "pipeline": ["quantizer", "codec"], "quantizer_config": dict(cfg),
                "codec_config": {"codec_type": "rans"}, "backend": "generic",
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
    p, c, pair = make_pair(ctl)
    pair.delay_s = 0.05
    comp = p._get_compressor()
    seen = []
    orig = comp.update_controller
    comp.update_controller = lambda rid, ms: (seen.append((rid, ms)), orig(rid, ms))
    handoff(p, c)
    assert seen == []  # nothing applied from the transport thread
    time.sleep(0.1)
    p.get_finished(set())
    assert [r for r, _ in seen] == ["r1"] and seen[0][1] >= 50.0
    assert comp.get_controller_stats()["bandit_states"] == 1 and not p._ctl_wait


def test_default_mode_handoff_on_cpu():
    """compression "default" on CPU caches: the adapter's generic twin of the
    fused path compresses, the consumer decodes into its own block ids."""
    p, c, pair = make_pair("default")
    pc, cc = handoff(p, c)
    assert pair.messages == 1
    for name in pc:
        a = pc[name][:, [5, 1, 7]].float().flatten()
        b = cc[name][:, [2, 6, 0]].float().flatten()
        assert float(torch.nn.functional.cosine_similarity(a, b, dim=0)) > 0.9


def test_head_count_mismatch_is_a_failed_load():
    """A message built for another per-rank head count (producer and
    consumer at different TP sizes) is not decoded: the load fails with a
    message that names the cause, and the blocks go to vLLM's policy."""
    import logging
    seen = []

    class Keep(logging.Handler):
        def emit(self, record):
            seen.append(record.getMessage())
    log = logging.getLogger("kvserve_hpdps_b200")
    h = Keep(level=logging.ERROR)
    log.addHandler(h)
    p, c, pair = make_pair("default")
    c._num_kv_heads = H // 2
    try:
        pc, cc = handoff(p, c)
    finally:
        log.removeHandler(h)
    assert any("heterogeneous TP" in m for m in seen)
    assert c.get_block_ids_with_load_errors() == {2, 6, 0}
    name = next(iter(cc))  # nothing of the producer's KV was written
    assert not torch.equal(cc[name][:, [2, 6, 0]], pc[name][:, [5, 1, 7]])


def test_compressed_handoff_with_blocks_outer_caches():
    """FlashInfer-layout caches ([num_blocks, 2, bs, H, D], what vLLM
    allocates on B200): the whole-tensor compressors get [L, 2, blocks, ...],
    so keys and values are quantized as keys and values, and the consumer
    writes each plane back into its own half of the blocks.  Keys and values
    have scales 100x apart, which a K/V mix-up would not survive."""
    p, c, pair = make_pair("default")
    g = torch.Generator().manual_seed(3)

    def fi_caches(fill):
        out = {}
        for l in range(L):
            t = torch.zeros(8, 2, BS, H, D)
            if fill:
                t[:, 0] = 10.0 * torch.randn(8, BS, H, D, generator=g)
                t[:, 1] = 0.1 * torch.randn(8, BS, H, D, generator=g)
            out[f"model.layers.{l}.self_attn.attn"] = t.to(torch.bfloat16)
        return out
    pc, cc = fi_caches(True), fi_caches(False)
    p.register_kv_caches(pc)
    c.register_kv_caches(cc)
    p.bind_connector_metadata(meta_for("r1", "tid-1", 48, [5, 1, 7]))
    for name in sorted(pc, key=layer_index):
        p.save_kv_layer(name, pc[name], None)
    p.wait_for_save()
    c.bind_connector_metadata(meta_for("d1", "tid-1", 48, [2, 6, 0]))
    c.start_load_kv(None)
    assert pair.messages == 1
    for name in pc:
        for plane in (0, 1):
            a = pc[name][[5, 1, 7], plane].float().flatten()
            b = cc[name][[2, 6, 0], plane].float().flatten()
            # 2-bit values of most heads keep cosine ~0.87 on Gaussian data
            assert float(torch.nn.functional.cosine_similarity(a, b, dim=0)) > 0.8, (name, plane)
            assert 0.5 < float(b.norm() / a.norm()) < 2.0, (name, plane)


def test_overlap_modes_are_normalized(monkeypatch):
    from kvserve_hpdps_b200.connector.compressed_kv_connector import normalize_overlap_mode
    assert [normalize_overlap_mode(m) for m in ("off", "stream", "tq", "full", "FULL", None,
                                                "bogus")] == \
        ["off", "stream", "off", "off", "off", "off", "off"]
    monkeypatch.setenv("KVSERVE_OVERLAP_MODE", "tq")
    p, _, _ = make_pair(None)
    assert p._overlap_mode == "off"


def test_paged_send_statistics_with_a_stand_in_compressor(monkeypatch):
    """The producer's paged compressed branch (GPU caches in production):
    the statistics entry is queued before the send, completed by the
    transport's report with the bytes that crossed, and taken back when the
    compressor sends nothing (its message then goes out raw)."""
    p, c, pair = make_pair(None)

    class CudaLike(torch.Tensor):  # a CPU tensor the branch takes for a CUDA cache
        @property
        def is_cuda(self):
            return True

    class Comp:
        controller_mode = False
        send = True

        def supports_paged(self):
            return True

        def send_paged_requests(self, tr, tid, names, layers, ids, reqs, member_tids=None):
            if not self.send:
                return None
            body = torch.zeros(1000, dtype=torch.uint8)
            tr.send_bundle(tid, names, {"m": 1}, [body], [], member_tids=member_tids)
            return {"original_size": 1, "wire_nbytes": 1000}

    comp = Comp()
    p._get_compressor = lambda: comp
    pc = {n: t.as_subclass(CudaLike) for n, t in caches(8, 1).items()}
    p.bind_connector_metadata(meta_for("r1", "tid-p", 40, [5, 1, 7]))
    p._layer_refs = dict(pc)
    p.wait_for_save()
    st = p.get_kv_connector_stats()
    assert st.data["original_bytes"] == [L * 2 * 40 * H * D * 2]
    assert st.data["wire_bytes"] == [1000] and not p._sent_orig
    # nothing sent by the compressor: the entry is taken back and the raw
    # message is recorded as raw
    import kvserve_hpdps_b200.connector.compressed_kv_connector as mod
    monkeypatch.setattr(mod, "extract_kv_from_layer_by_blocks",
                        lambda layer, ids: layer.as_subclass(torch.Tensor)[:, ids])
    comp.send = False
    p.bind_connector_metadata(meta_for("r2", "tid-q", 40, [5, 1, 7]))
    p._layer_refs = dict(pc)
    p.wait_for_save()
    st = p.get_kv_connector_stats()
    raw = L * 2 * 3 * BS * H * D * 2
    assert st.data["original_bytes"] == [raw] and st.data["wire_bytes"] == [raw]
    assert not p._sent_orig


def test_layer_chunked_request_of_a_tp_rank_through_the_connector(monkeypatch):
    """The long-request path at a TP rank (config 4's shape, scaled down):
    rank 1 of 4 of a Qwen2.5-32B-style model (2 KV heads per rank) sends a
    request above the chunking threshold, so the message is a
    ``manager_chunks`` body of layer chunks; the consumer rebuilds every
    layer into its own blocks."""
    import kvserve_hpdps_b200.compression.pipeline_manager as PM
    monkeypatch.setattr(PM, "CHUNK_THRESHOLD_BYTES", 64 << 10)
    layers, heads = 12, 2
    spec = {"enabled": True, "pipeline": ["transformer", "quantizer", "codec"],
            "transformer_config": {"seed": 0x3333}, "backend": "generic",
            "quantizer_config": {"hybrid_ratio": 0.3, "high_key_max_value": 16,
                                 "high_value_max_value": 16, "low_key_max_value": 12,
                                 "low_value_max_value": 12, "axis_key": "channel",
                                 "axis_value": "token", "split_type": "head"},
            "codec_config": {"codec_type": "rans"}}

    def cfg(producer):
        c = vllm_config(producer, spec)
        c.model_config = SimpleNamespace(
            get_num_kv_heads=lambda pc: heads, get_head_size=lambda: D,
            get_num_layers=lambda pc: layers, model="/models/Qwen2.5-32B-Instruct",
            hf_text_config=SimpleNamespace(num_hidden_layers=layers), use_mla=False)
        return c
    pair = FakeTransportPair()
    p = CompressedKVConnector(cfg(True), KVConnectorRole.WORKER)
    c = CompressedKVConnector(cfg(False), KVConnectorRole.WORKER)
    for conn in (p, c):
        conn._tp_rank, conn._tp_size, conn._compressor = 1, 4, None
    p.attach_transport(pair.producer())
    c.attach_transport(pair.consumer())
    g = torch.Generator().manual_seed(7)
    pc = {f"model.layers.{l}.self_attn.attn":
          torch.randn(2, 8, BS, heads, D, generator=g).to(torch.bfloat16) for l in range(layers)}
    cc = {k: torch.zeros_like(v) for k, v in pc.items()}
    p.register_kv_caches(pc)
    c.register_kv_caches(cc)
    p.bind_connector_metadata(meta_for("r1", "tid-long", 60, [5, 1, 7, 2]))
    for name in sorted(pc, key=layer_index):
        p.save_kv_layer(name, pc[name], None)
    p.wait_for_save()
    payload = pair.inbox["tid-long"][0][1]
    assert payload["meta"]["body_mode"] == "manager_chunks" and len(payload["body_chunks"]) == 2
    c.bind_connector_metadata(meta_for("d1", "tid-long", 60, [0, 3, 6, 4]))
    c.start_load_kv(None)
    assert c.get_block_ids_with_load_errors() == set()
    for name in pc:
        a = pc[name][:, [5, 1, 7, 2]].float().flatten()
        b = cc[name][:, [0, 3, 6, 4]].float().flatten()
        assert float(torch.nn.functional.cosine_similarity(a, b, dim=0)) > 0.97


def test_late_transport_reports_still_find_their_statistics_entry(monkeypatch):
    """A transport may report a message sent just after the producer's wait
    for it returned: the entry stays until its time-to-live has passed, then
    unreported entries (refused messages) are dropped."""
    import kvserve_hpdps_b200.connector.compressed_kv_connector as mod
    p, _, _ = make_pair(None)
    p._expect_sent("t-late", 4000)
    p._retire_sent_entries(["t-late"])        # the step's wait returned
    p._on_sent("t-late", ["t-late"], 2.0, nbytes=1000)  # ...then the report
    st = p.get_kv_connector_stats()
    assert st.data["original_bytes"] == [4000] and st.data["wire_bytes"] == [1000]
    p._expect_sent("t-refused", 4000)          # never reported
    monkeypatch.setattr(mod, "STATS_ENTRY_TTL_S", 0.0)
    p._retire_sent_entries(["t-refused"])
    p._retire_sent_entries([])
    assert "t-refused" not in p._sent_orig


@pytest.mark.parametrize("compression", [None, "default"])
def test_soak_with_random_failures(compression, monkeypatch):
    """Thirty steps of one to three requests of random lengths through a
    producer/consumer pair, with messages dropped, refused or delayed at
    random: every request either arrives intact (raw) or close (compressed)
    in its consumer blocks, or its blocks are reported to vLLM's load-failure
    policy in that step; nothing accumulates in the connectors."""
    import random

    import kvserve_hpdps_b200.connector.compressed_kv_connector as mod
    monkeypatch.setattr(mod, "LOAD_TIMEOUT_S", 0.15)
    monkeypatch.setattr(mod, "STATS_ENTRY_TTL_S", 0.0)
    rng = random.Random(7 if compression else 8)
    p, c, pair = make_pair(compression)
    nb = 64
    pc, cc = caches(nb, 11), caches(nb, 12)
    p.register_kv_caches(pc)
    c.register_kv_caches(cc)
    loaded = failed = 0
    for step in range(30):
        free_p, free_c = list(range(nb)), list(range(nb))
        rng.shuffle(free_p)
        rng.shuffle(free_c)
        reqs = []
        for i in range(rng.randint(1, 3)):
            ntok = rng.randint(1, 80)
            k = -(-ntok // BS)
            reqs.append((f"s{step}r{i}", f"t{step}-{i}", ntok,
                         [free_p.pop() for _ in range(k)], [free_c.pop() for _ in range(k)]))
        fault = rng.random()
        if fault < 0.15:
            pair.drop_next = 1
        elif fault < 0.3:
            pair.refuse_next = 1
        pm, cm = CompressedKVConnectorMetadata(), CompressedKVConnectorMetadata()
        for rid, tid, ntok, pb, cb in reqs:
            pm.add_request(rid, tid, list(range(ntok)), pb, BS)
            cm.add_request("d" + rid, tid, list(range(ntok)), cb, BS)
        p.bind_connector_metadata(pm)
        for name in sorted(pc, key=layer_index):
            p.save_kv_layer(name, pc[name], None)
        p.wait_for_save()
        c.bind_connector_metadata(cm)
        c.start_load_kv(None)
        bad = c.get_block_ids_with_load_errors()
        for rid, tid, ntok, pb, cb in reqs:
            if set(cb) <= bad:
                failed += 1
                continue
            assert not set(cb) & bad, (step, rid)
            for name in pc:
                a, b = pc[name][:, pb].float(), cc[name][:, cb].float()
                if compression is None:
                    assert torch.equal(a, b), (step, rid)
                else:
                    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0)
                    assert float(cos) > 0.9, (step, rid, float(cos))
            loaded += 1
        c.get_kv_connector_stats()
        p.get_kv_connector_stats()
    assert loaded > 20 and failed > 0
    p._retire_sent_entries([])
    assert not p._sent_orig and not p._stats_wait and not p._save_times
    assert not c._worker_received and not c._partial and not c._load_errors



def test_late_messages_of_failed_loads_are_released(monkeypatch):
    """A message that arrives after its request's load timed out (the
    blocks went to vLLM's policy) is not queued for good: it is released on
    arrival, and a message already queued for a failed request is dropped at
    the next step."""
    import time
    import kvserve_hpdps_b200.connector.compressed_kv_connector as mod
    monkeypatch.setattr(mod, "LOAD_TIMEOUT_S", 0.1)
    p, c, pair = make_pair(None)
    released = []
    pair_cons = c._transport
    pair_cons.release = lambda payload, dev=None: released.append(payload)
    pair.delay_s = 0.4
    handoff(p, c)                      # the message comes after the step gave up
    assert c.get_block_ids_with_load_errors() == {2, 6, 0}
    time.sleep(0.5)
    c.bind_connector_metadata(CompressedKVConnectorMetadata())
    c.start_load_kv(None)              # drained at the next step: released at once
    assert len(released) == 1 and not c._worker_received


def test_unclaimed_messages_are_released_after_their_ttl(monkeypatch):
    """KV for a transfer id the decode engine never schedules (its request
    never reached it) does not hold its ring space for good."""
    import kvserve_hpdps_b200.connector.compressed_kv_connector as mod
    p, c, pair = make_pair(None)
    released = []
    c._transport.release = lambda payload, dev=None: released.append(payload)
    pc = caches(8, 1)
    p.register_kv_caches(pc)
    c.register_kv_caches(caches(8, 2))
    p.bind_connector_metadata(meta_for("r1", "orphan", 40, [5, 1, 7]))
    for name in sorted(pc, key=layer_index):
        p.save_kv_layer(name, pc[name], None)
    p.wait_for_save()
    c.bind_connector_metadata(CompressedKVConnectorMetadata())
    c.start_load_kv(None)               # arrives; nobody claims it yet
    assert "orphan" in c._worker_received and not released
    monkeypatch.setattr(mod, "UNCLAIMED_TTL_S", 0.0)
    c.start_load_kv(None)
    assert not c._worker_received and len(released) == 1


def test_swept_group_record_is_released_once_and_fails_its_late_members(monkeypatch):
    """A grouped message decoded for one member while another member is
    never scheduled: after twice the load timeout its ring space goes back
    (once, whichever cleanup comes first), and the member that shows up
    later fails its load cleanly instead of decoding released memory."""
    import kvserve_hpdps_b200.connector.compressed_kv_connector as mod
    monkeypatch.setattr(mod, "LOAD_TIMEOUT_S", 0.05)
    p, c, pair = make_pair(None)
    released = []
    c._transport.release = lambda payload, dev=None: released.append(id(payload))
    pc = caches(8, 1)
    c.register_kv_caches(caches(8, 2))
    raw = torch.stack([pc[n][:, [5, 1, 7]] for n in sorted(pc, key=layer_index)], 0)
    payload = {"__bundle__": True, "meta": {"metadata": {"member_tids": ["ga", "gb"]}},
               "body_chunks": [], "aux_tensors": []}
    # a grouped record as the transport delivers it; decoding fails here (no
    # real compressed body), which is enough to exercise the bookkeeping
    pair.inbox["ga"].append((["__compressed__"] + sorted(pc, key=layer_index), payload))
    c.bind_connector_metadata(meta_for("da", "ga", 40, [2, 6, 0]))
    c.start_load_kv(None)
    assert "gb" in c._worker_received and len(c._partial) == 1
    import time
    time.sleep(0.15)
    c.bind_connector_metadata(CompressedKVConnectorMetadata())
    c.start_load_kv(None)          # sweep: released once, gb abandoned
    monkeypatch.setattr(mod, "UNCLAIMED_TTL_S", 0.0)
    c.start_load_kv(None)          # the unclaimed cleanup finds nothing left to release
    assert released == [id(payload)] and not c._worker_received and not c._partial
    c.get_block_ids_with_load_errors()
    c.bind_connector_metadata(meta_for("db", "gb", 40, [3, 4, 5]))
    c.start_load_kv(None)          # gb scheduled late: times out cleanly, reported
    assert c.get_block_ids_with_load_errors() == {3, 4, 5}
    assert released == [id(payload)]
    del raw
