"""Wire-level interoperability with the reference implementation (installed
in ``baseline/_ref``; skipped without it): a message compressed by either
framework's quantizer pipeline and carried in its wire envelope is restored
and decompressed by the other into the same KV.  Runs in a child process so
that the reference package never enters this test session."""

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

CODE = r"""
import sys
sys.path.insert(0, ROOT)
sys.path.insert(0, REF)
import torch
from kvserve_hpdps_b200.compression import wire as OW
from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter as Ours
from kvserve_v1.compression import wire as RW
from kvserve_v1.compression.manager import KVCompressionAdapter as Ref
L, T, H, D = 4, 256, 4, 128
g = torch.Generator().manual_seed(0)
x = torch.randn((L, 2, 1, T, H, D), generator=g)
x[:, 0, ..., :4] *= 12
x = x.to(torch.bfloat16)
qc = {"model_name": "Qwen2.5-7B-Instruct", "hybrid_ratio": 0.3, "high_key_max_value": 16,
      "high_value_max_value": 16, "low_key_max_value": 12, "low_value_max_value": 16,
      "axis_key": "channel", "axis_value": "token", "split_type": "head"}
ours = Ours({"enabled": True, "pipeline": ["quantizer"], "backend": "generic",
             "quantizer_config": qc, "min_compress_size": 0}, H, D,
            model_name="Qwen2.5-7B-Instruct", num_layers=28)
ref = Ref({"enabled": True, "pipeline": ["quantizer"], "quantizer_config": qc}, H, D,
          model_name="Qwen2.5-7B-Instruct")
cd = ours.compress(x, "a")
w = OW.build_wire(cd, 512 << 20)
by_ref = ref.decompress(RW.restore_from_wire(RW.CompressedWire(w.meta, w.body_chunks,
                                                               w.aux_tensors)))
assert torch.equal(by_ref.reshape(-1), ours.decompress(cd).reshape(-1)), "ours -> reference"
rc = ref.compress(x, "b")
rw = RW.build_wire(rc, 512 << 20)
by_ours = ours.decompress(OW.restore_from_wire(OW.CompressedWire(rw.meta, rw.body_chunks,
                                                                 rw.aux_tensors)))
assert torch.equal(by_ours.reshape(-1), ref.decompress(rc).reshape(-1)), "reference -> ours"
assert torch.equal(cd.compressed_tensor.view(torch.uint8).reshape(-1),
                   rc.compressed_tensor.view(torch.uint8).reshape(-1)), "bodies"
# layer-chunked messages (manager_chunks body mode): the size threshold is
# lowered on our side and the reference's chunked path is called directly
from kvserve_hpdps_b200.compression import pipeline_manager as PM
L2 = 20
x2 = torch.randn((L2, 2, 1, 64, H, D), generator=g).to(torch.bfloat16)
PM.CHUNK_THRESHOLD_BYTES = 1024
cd2 = ours.compress(x2, "c")
assert cd2.is_chunked and len(cd2.chunks) == 3
w2 = OW.build_wire(cd2, 512 << 20)
assert w2.meta["body_mode"] == "manager_chunks"
r2 = ref.decompress(RW.restore_from_wire(RW.CompressedWire(w2.meta, w2.body_chunks,
                                                           w2.aux_tensors)))
assert torch.equal(r2.reshape(-1), ours.decompress(cd2).reshape(-1)), "chunked ours -> reference"
rc2 = ref._manager._compress_all_layers_chunked(
    x2, "d", {"original_dtype": "bfloat16", "original_shape": list(x2.shape)}, chunk_size=8)
rw2 = RW.build_wire(rc2, 512 << 20)
assert rw2.meta["body_mode"] == "manager_chunks"
o2 = ours.decompress(OW.restore_from_wire(OW.CompressedWire(rw2.meta, rw2.body_chunks,
                                                            rw2.aux_tensors)))
assert torch.equal(o2.reshape(-1), ref.decompress(rc2).reshape(-1)), "chunked reference -> ours"
print("INTEROP OK")
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_wire_messages_cross_between_the_frameworks():
    code = CODE.replace("ROOT", repr(ROOT)).replace("REF", repr(REF))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd="/tmp" if os.path.isdir("/tmp") else ROOT)
    assert out.returncode == 0 and "INTEROP OK" in out.stdout, out.stderr[-3000:]


CTL = r"""
import json, sys
sys.path.insert(0, ROOT)
sys.path.insert(0, REF)
from kvserve_hpdps_b200.controller.analytical_model import AnalyticalModel
from kvserve_hpdps_b200.controller.online_controller import OnlineController as Ours
from kvserve_hpdps_b200.controller.profile_library import ProfileLibrary as OursLib
from kvserve_hpdps_b200.offline.library_export import build_library, write_library
from kvserve_hpdps_b200.offline.search_space import Candidate
from kvserve_v1.compression.controller.online_controller import OnlineController as Ref
from kvserve_v1.compression.controller.profile_library import ProfileLibrary as RefLib
evals = []
for c, acc, cr, s in [(Candidate(0.0, 16, 16, 8, 6), 0.995, 3.5, 30000.0),
                      (Candidate(0.3, 16, 12, 8, 6), 0.985, 4.6, 24000.0),
                      (Candidate(0.8, 12, 8, 6, 4), 0.97, 6.0, 20000.0),
                      (Candidate(1.0, 12, 8, 6, 4), 0.93, 7.4, 16000.0)]:
    evals.append({"candidate": c.key(), "config": c.quantizer_config(), "accuracy": acc,
                  "compression_ratio": cr, "harmonic_speed_mbps": s})
path = TMP + "/lib.json"
write_library(path, build_library(evals, "Qwen2.5-7B-Instruct"))
ours = Ours(OursLib(path), epsilon=0.0, model=AnalyticalModel(reference_transfer_term=True))
ref = Ref(RefLib(path), epsilon=0.0)
n = 0
compared = set()
for V in (64e6, 470e6, 2e9):
    for B in (2.0, 10.0, 50.0, 150.0, 400.0, 1000.0, 3000.0, 1e6):
        for slo in (50.0, 500.0, 1e9):
            for acc in (0.9, 0.96, 0.99, 0.999):
                po, co = ours.select_profile(V, B, 10.0, slo, acc)
                pr, cr_ = ref.select_profile(V, B, 10.0, slo, acc)
                ido = None if po is None else po.profile_id
                idr = None if pr is None else pr.profile_id
                assert ido == idr, (V, B, slo, acc, ido, idr)
                for k in ("bucket_id", "interval_id", "profile_id", "action", "num_candidates",
                          "T_hat", "T_eff", "delta_bar", "baseline_latency", "speedup_predicted"):
                    if k in cr_:
                        a, b = co.get(k), cr_[k]
                        assert a == b or (isinstance(b, float) and abs(a - b) <= 1e-9 * max(1, abs(b))), \
                            (k, co, cr_)
                        compared.add(k)
                if po is not None:
                    t = 5.0 + (n % 7)
                    ours.update(co, t)
                    ref.update(cr_, t)
                n += 1
so, sr = ours.get_statistics(), ref.get_statistics()
for k in ("total_decisions", "exploit_count", "explore_count", "no_compression_count"):
    assert so[k] == sr[k], (k, so, sr)
assert {"profile_id", "T_hat", "T_eff", "delta_bar"} <= compared, compared
# bandit state files cross both ways and keep learning identically
ref.save_state(TMP + "/ref_state.json")
ours.save_state(TMP + "/ours_state.json")
o2 = Ours(OursLib(path), epsilon=0.0, model=AnalyticalModel(reference_transfer_term=True))
r2 = Ref(RefLib(path), epsilon=0.0)
o2.load_state(TMP + "/ref_state.json")
r2.load_state(TMP + "/ours_state.json")
po, co = o2.select_profile(470e6, 50.0, 10.0, 1e9, 0.96)
pr, cr_ = r2.select_profile(470e6, 50.0, 10.0, 1e9, 0.96)
assert po is not None and pr is not None and po.profile_id == pr.profile_id
assert abs(co["delta_bar"] - cr_["delta_bar"]) < 1e-9 and co["delta_bar"] != 0.0, (co, cr_)
o2.update(co, 42.0)
r2.update(cr_, 42.0)
b, i, pid = co["bucket_id"], co["interval_id"], co["profile_id"]
so, sr = o2.bandit.get_stats(b, i, pid), r2.bandit.get_stats(b, i, pid)
assert so[0] == sr[0] and abs(so[1] - sr[1]) < 1e-9, (so, sr)
print("CONTROLLER OK", n)
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_controller_decisions_match_the_reference(tmp_path):
    """Same library, same requests: both controllers (with the reference's
    transfer term selected here) pick the same profile, with the same bucket,
    interval and predicted latency, and keep the same statistics."""
    code = CTL.replace("ROOT", repr(ROOT)).replace("REF", repr(REF)) \
        .replace("TMP", repr(str(tmp_path)))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd=str(tmp_path))
    assert out.returncode == 0 and "CONTROLLER OK" in out.stdout, \
        (out.stdout[-1500:] + out.stderr[-3000:])


PARTS = r"""
import sys, types
sys.path.insert(0, ROOT)
sys.path.insert(0, REF)
# the reference's transform module imports its FWHT extension at import time;
# only its sign generation (plain torch) is called here
sys.modules.setdefault("fast_hadamard_transform", types.ModuleType("fast_hadamard_transform"))
import torch
from kvserve_hpdps_b200.compression import wire as OW
from kvserve_hpdps_b200.compression.head_scores import slice_for_tp
from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter as Ours
from kvserve_hpdps_b200.compression.quantizer import KVServeQuantizer as OQ
from kvserve_hpdps_b200.compression.transformer import HadamardTransform as OH
from kvserve_v1.compression import wire as RW
from kvserve_v1.compression.manager import KVCompressionAdapter as Ref
from kvserve_v1.compression.quantizer.kvserve_quantizer import KVServeQuantizer as RQ
from kvserve_v1.compression.transformer.hadamard_func import HadamardTransform as RH
# Rademacher signs
for seed in (0x3333, 0xC0FEBABE):
    for layer in (0, 5, 27):
        a = OH(seed).get_rademacher_signs(layer, 8, 128, torch.device("cpu"), torch.float32)
        b = RH(seed).get_rademacher_signs(layer, 8, 128, torch.device("cpu"), torch.float32)
        assert torch.equal(a, b), ("signs", seed, layer)
# hybrid head / layer masks and their TP slices
for model in ("Qwen2.5-7B-Instruct", "Llama-3.1-8B-Instruct", "Qwen2.5-32B-Instruct"):
    for hr in (0.0, 0.3, 0.5, 0.8, 1.0):
        o, r = OQ(model_name=model, hybrid_ratio=hr), RQ(model_name=model, hybrid_ratio=hr)
        assert torch.equal(o.head_scores_mask, r.head_scores_mask), ("head mask", model, hr)
        assert torch.equal(o.layer_scores_mask, r.layer_scores_mask), ("layer mask", model, hr)
        H = r.head_scores_mask.shape[1]
        for tp in (2,):
            for rank in range(tp):
                rt = RQ(model_name=model, hybrid_ratio=hr, tensor_parallel_size=tp, tp_rank=rank)
                got = slice_for_tp(o.head_scores_mask, H // tp, rank, tp)
                assert torch.equal(got, rt._get_tp_head_scores_mask(H // tp)), ("tp", model, hr, rank)
# chunked wire bodies (byte_chunks) in both directions
L, T, H, D = 2, 128, 4, 128
x = torch.randn((L, 2, 1, T, H, D), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
qc = {"model_name": "Qwen2.5-7B-Instruct", "hybrid_ratio": 0.5, "axis_key": "channel",
      "axis_value": "token", "split_type": "head"}
ours = Ours({"enabled": True, "pipeline": ["quantizer"], "backend": "generic",
             "quantizer_config": qc, "min_compress_size": 0}, H, D,
            model_name="Qwen2.5-7B-Instruct", num_layers=28)
ref = Ref({"enabled": True, "pipeline": ["quantizer"], "quantizer_config": qc}, H, D,
          model_name="Qwen2.5-7B-Instruct")
cd = ours.compress(x, "a")
w = OW.build_wire(cd, 4096)
assert w.meta["body_mode"] == "byte_chunks" and len(w.body_chunks) > 1
by_ref = ref.decompress(RW.restore_from_wire(RW.CompressedWire(w.meta, w.body_chunks,
                                                               w.aux_tensors)))
assert torch.equal(by_ref.reshape(-1), ours.decompress(cd).reshape(-1)), "chunked ours -> ref"
rw = RW.build_wire(ref.compress(x, "b"), 4096)
assert rw.meta["body_mode"] == "byte_chunks"
by_ours = ours.decompress(OW.restore_from_wire(OW.CompressedWire(rw.meta, rw.body_chunks,
                                                                 rw.aux_tensors)))
assert torch.equal(by_ours.reshape(-1), by_ref.reshape(-1)), "chunked ref -> ours"
# the hybrid quantizer itself: codes, metadata and reconstruction per layer
def _same(a, b):
    if torch.is_tensor(a):
        return torch.is_tensor(b) and a.shape == b.shape and torch.equal(a, b)
    if isinstance(a, dict):
        return isinstance(b, dict) and a.keys() == b.keys() and all(_same(a[k], b[k]) for k in a)
    return a == b
gq = torch.Generator().manual_seed(6)
for split in ("head", "layer"):
    for ak, av in (("channel", "token"), ("token", "token"), ("tensor", "channel")):
        kw = dict(model_name="Qwen2.5-7B-Instruct", hybrid_ratio=0.5, high_key_max_value=16,
                  high_value_max_value=12, low_key_max_value=8, low_value_max_value=6,
                  axis_key=ak, axis_value=av, split_type=split)
        oq, rq = OQ(**kw), RQ(**kw)
        for layer in (0, 13, 27):
            x = (torch.randn(2, 5, 16, 4, 128, generator=gq) * 3).to(torch.bfloat16)
            qo, mo = oq.quantize(layer, x)
            qr, mr = rq.quantize(layer, x)
            assert torch.equal(qo, qr) and _same(mo, mr), ("quantize", split, ak, av, layer)
            assert torch.equal(oq.dequantize(layer, qo, mo), rq.dequantize(layer, qr, mr)), \
                ("dequantize", split, ak, av, layer)
# paged KV block utilities: both cache layouts, shuffled and repeated block ids
from kvserve_hpdps_b200.utils import kv_utils as OK_
from kvserve_v1.utils import kv_utils as RK_
tok = list(range(45))
assert torch.equal(OK_.make_slot_mapping(tok, [7, 2, 9], 16), RK_.make_slot_mapping(tok, [7, 2, 9], 16))
gk = torch.Generator().manual_seed(4)
for shape in ((2, 10, 16, 4, 128), (10, 2, 16, 4, 128)):
    layer = torch.randn(shape, generator=gk).to(torch.bfloat16)
    ids = [7, 2, 9, 0]
    a, b = OK_.extract_kv_from_layer_by_blocks(layer, ids), RK_.extract_kv_from_layer_by_blocks(layer, ids)
    assert torch.equal(a, b), ("extract", shape)
    l1, l2 = torch.zeros_like(layer), torch.zeros_like(layer)
    OK_.inject_kv_into_layer_by_blocks(l1, a, [3, 1, 8, 5])
    RK_.inject_kv_into_layer_by_blocks(l2, b, [3, 1, 8, 5])
    assert torch.equal(l1, l2), ("inject", shape)
    sm = OK_.make_slot_mapping(list(range(40)), [3, 1, 8], 16)
    x1 = OK_.extract_kv_from_layer(layer, sm) if shape[0] == 2 else None
    if x1 is not None:
        assert torch.equal(x1, RK_.extract_kv_from_layer(layer, sm)), "extract slots"
        m1, m2 = torch.zeros_like(layer), torch.zeros_like(layer)
        OK_.inject_kv_into_layer(m1, x1, sm)
        RK_.inject_kv_into_layer(m2, x1, sm)
        assert torch.equal(m1, m2), "inject slots"
print("PARTS OK")
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_signs_masks_and_chunked_wire_match_the_reference(tmp_path):
    """Rademacher signs, hybrid head/layer masks (and their TP slices) equal
    the reference's, and chunked wire bodies cross in both directions."""
    code = PARTS.replace("ROOT", repr(ROOT)).replace("REF", repr(REF))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd=str(tmp_path))
    assert out.returncode == 0 and "PARTS OK" in out.stdout, \
        (out.stdout[-1500:] + out.stderr[-3000:])


SCHED = r"""
import sys
from types import SimpleNamespace as NS
sys.path.insert(0, ROOT)
sys.path.insert(0, REF)
import os
os.environ["KVSERVE_TRANSPORT"] = "fake"
from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
from kvserve_hpdps_b200.connector.compressed_kv_connector import CompressedKVConnector as Ours
from kvserve_v1.connector.compressed_kv_connector import CompressedKVConnector as Ref

def cfg(producer):
    mc = NS(get_num_kv_heads=lambda pc: 4, get_head_size=lambda: 128,
            get_num_layers=lambda pc: 2, model="/models/Qwen2.5-7B-Instruct",
            hf_text_config=NS(num_hidden_layers=2), use_mla=False)
    kv = NS(is_kv_producer=producer, kv_ip="127.0.0.1", kv_port=29999, kv_role="kv_both",
            kv_connector_extra_config={"compression": None}, kv_parallel_size=2, kv_rank=0)
    return NS(kv_transfer_config=kv, cache_config=NS(block_size=16), model_config=mc,
              parallel_config=NS())

def meta_rows(m):
    return [(r.request_id, r.transfer_id, list(r.token_ids), list(r.block_ids),
             r.slot_mapping.tolist()) for r in m.requests]

def script(conn, producer):
    out = []
    reqs = {"r": NS(request_id="r", prompt_token_ids=list(range(50)),
                    kv_transfer_params={"transfer_id": "T9"}, all_token_ids=list(range(51))),
            "c": NS(request_id="c", prompt_token_ids=list(range(40)),
                    kv_transfer_params={"transfer_id": "TC"}, all_token_ids=list(range(40))),
            "n": NS(request_id="n", prompt_token_ids=list(range(20)), kv_transfer_params=None,
                    all_token_ids=list(range(20))),
            "p": NS(request_id="p", prompt_token_ids=list(range(33)),
                    kv_transfer_params={"transfer_id": "TP"}, all_token_ids=list(range(35))),
            "q": NS(request_id="q", prompt_token_ids=list(range(40)),
                    kv_transfer_params={"transfer_id": "TQ"}, all_token_ids=list(range(40)))}
    for rid, r in reqs.items():
        out.append(("matched", rid, conn.get_num_new_matched_tokens(r, 0),
                    conn.get_num_new_matched_tokens(r, 16)))
    blocks = {"r": [3, 4, 5, 6], "c": [1, 2], "n": [7, 8], "p": [10, 11, 12], "q": [16]}
    for rid, r in reqs.items():
        n_ext = 0 if producer else max(0, len(r.prompt_token_ids) - 1)
        conn.update_state_after_alloc(r, NS(get_block_ids=lambda b=blocks[rid]: (b,)), n_ext)
    empty = NS(req_ids=[], num_computed_tokens=[], new_block_ids=[], resumed_req_ids=set())
    new = lambda rid, n0=0: NS(req_id=rid, prompt_token_ids=reqs[rid].prompt_token_ids,
                               block_ids=(blocks[rid],), num_computed_tokens=n0)
    so1 = NS(scheduled_new_reqs=[new("r"), new("c"), new("n"), new("q")],
             num_scheduled_tokens={"r": 50, "c": 32, "n": 20, "q": 16},
             scheduled_cached_reqs=empty)
    out.append(("step1", meta_rows(conn.build_connector_meta(so1))))
    cached = NS(req_ids=["c"], num_computed_tokens=[32], new_block_ids=[([9],)],
                resumed_req_ids=set())
    so2 = NS(scheduled_new_reqs=[], num_scheduled_tokens={"c": 8}, scheduled_cached_reqs=cached)
    out.append(("step2", meta_rows(conn.build_connector_meta(so2))))
    # resumed after preemption: the producer's chunked prefill "q" restarts in new
    # blocks; the consumer's "p" (never scheduled before) loads into its new blocks
    rid3 = "q" if producer else "p"
    resumed = NS(req_ids=[rid3], num_computed_tokens=[0 if producer else 32],
                 new_block_ids=[([20, 21, 22],)], resumed_req_ids={rid3})
    so3 = NS(scheduled_new_reqs=[], num_scheduled_tokens={rid3: 40 if producer else 1},
             scheduled_cached_reqs=resumed)
    out.append(("step3", meta_rows(conn.build_connector_meta(so3))))
    out.append(("finished", conn.request_finished(reqs["r"], blocks["r"])))
    return out

for producer in (True, False):
    a = script(Ours(cfg(producer), KVConnectorRole.SCHEDULER), producer)
    b = script(Ref(cfg(producer), KVConnectorRole.SCHEDULER), producer)
    for x, y in zip(a, b):
        assert x == y, ("producer" if producer else "consumer", x, y)
    assert len(a) == len(b)
print("SCHEDULER OK")
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_scheduler_side_matches_the_reference(tmp_path):
    """Producer and consumer scheduler-side connectors on the same scripted
    steps (full prompt, chunked prefill over two steps, a request without a
    transfer id, a request resumed after preemption) build the same request
    metadata as the reference's connector: ids, tokens, blocks, slots.  (The
    steps are ones the reference accepts: its producer asserts that every
    scheduled cached request is a chunked prefill.)"""
    pytest.importorskip("vllm")
    code = SCHED.replace("ROOT", repr(ROOT)).replace("REF", repr(REF))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=900, cwd=str(tmp_path))
    assert out.returncode == 0 and "SCHEDULER OK" in out.stdout, \
        (out.stdout[-1500:] + out.stderr[-3000:])


SCHED_RANDOM = r"""
import random, sys
from types import SimpleNamespace as NS
sys.path.insert(0, ROOT)
sys.path.insert(0, REF)
import os
os.environ["KVSERVE_TRANSPORT"] = "fake"
from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
from kvserve_hpdps_b200.connector.compressed_kv_connector import CompressedKVConnector as Ours
from kvserve_v1.connector.compressed_kv_connector import CompressedKVConnector as Ref

BS = 16

def cfg(producer):
    mc = NS(get_num_kv_heads=lambda pc: 4, get_head_size=lambda: 128,
            get_num_layers=lambda pc: 2, model="/models/Qwen2.5-7B-Instruct",
            hf_text_config=NS(num_hidden_layers=2), use_mla=False)
    kv = NS(is_kv_producer=producer, kv_ip="127.0.0.1", kv_port=29999, kv_role="kv_both",
            kv_connector_extra_config={"compression": None}, kv_parallel_size=2, kv_rank=0)
    return NS(kv_transfer_config=kv, cache_config=NS(block_size=BS), model_config=mc,
              parallel_config=NS())

def rows(m):
    return [(r.request_id, r.transfer_id, list(r.token_ids), list(r.block_ids),
             r.slot_mapping.tolist()) for r in m.requests]

def producer_trace(seed):
    # chunked prefills interleaved over steps, some restarted after preemption
    rng = random.Random(seed)
    free = list(range(1000)); rng.shuffle(free)
    reqs, steps = {}, []
    for i in range(rng.randint(3, 8)):
        P = rng.randint(1, 150)
        cuts = sorted(rng.sample(range(1, P), min(P - 1, rng.randint(0, 3)))) if P > 1 else []
        reqs[f"r{i}"] = {"P": P, "chunks": [b - a for a, b in zip([0] + cuts, cuts + [P])],
                         "tid": None if rng.random() < 0.2 else f"T{seed}-{i}",
                         "start": rng.randint(0, 4)}
    state = {rid: {"done": 0, "k": 0, "blocks": 0} for rid in reqs}
    for step in range(12):
        new, cached, sched, resumed = [], [], {}, set()
        for rid, r in reqs.items():
            st = state[rid]
            if step < r["start"] or st["k"] >= len(r["chunks"]) or rng.random() < 0.3:
                continue
            restart = st["k"] > 0 and rng.random() < 0.15
            if restart:  # preempted: everything again, in new blocks
                st["done"], st["k"], st["blocks"] = 0, 0, 0
            n = r["chunks"][st["k"]]
            need = -(-(st["done"] + n) // BS) - st["blocks"]
            blocks = [free.pop() for _ in range(need)]
            if st["k"] == 0 and not restart:
                new.append((rid, blocks))
            else:
                cached.append((rid, st["done"], blocks))
                if restart:
                    resumed.add(rid)
            sched[rid] = n
            st["done"] += n; st["k"] += 1; st["blocks"] += need
        fin = [rid for rid in reqs if state[rid]["k"] >= len(reqs[rid]["chunks"])
               and rng.random() < 0.3 and not state[rid].get("fin")]
        for rid in fin:
            state[rid]["fin"] = True
        steps.append((new, cached, sched, resumed, fin))
    return reqs, steps

def play_producer(conn, reqs, steps):
    out = []
    R = {rid: NS(request_id=rid, prompt_token_ids=list(range(r["P"])),
                 kv_transfer_params={"transfer_id": r["tid"]} if r["tid"] else None,
                 all_token_ids=list(range(r["P"] + 1))) for rid, r in reqs.items()}
    for new, cached, sched, resumed, fin in steps:
        for rid, blocks in new:
            out.append(("matched", rid, conn.get_num_new_matched_tokens(R[rid], 0)))
            conn.update_state_after_alloc(R[rid], NS(get_block_ids=lambda b=blocks: (b,)), 0)
        so = NS(scheduled_new_reqs=[NS(req_id=rid, prompt_token_ids=R[rid].prompt_token_ids,
                                       block_ids=(b,), num_computed_tokens=0) for rid, b in new],
                num_scheduled_tokens=dict(sched),
                scheduled_cached_reqs=NS(req_ids=[c[0] for c in cached],
                                         num_computed_tokens=[c[1] for c in cached],
                                         new_block_ids=[(c[2],) for c in cached],
                                         resumed_req_ids=set(resumed)))
        out.append(("meta", rows(conn.build_connector_meta(so))))
        for rid in fin:
            out.append(("finished", rid, conn.request_finished(R[rid], [])))
    return out

def consumer_trace(seed):
    # new requests with a locally cached prefix, requests first seen resumed,
    # decode steps of loaded requests
    rng = random.Random(1000 + seed)
    free = list(range(1000)); rng.shuffle(free)
    reqs = {}
    for i in range(rng.randint(3, 8)):
        P = rng.randint(1, 150)
        pre = BS * rng.randint(0, max(0, (P - 1) // BS))
        reqs[f"d{i}"] = {"P": P, "pre": pre, "tid": None if rng.random() < 0.2 else f"U{seed}-{i}",
                         "kind": rng.choice(["new", "new", "resumed"]), "start": rng.randint(0, 3),
                         "blocks": [free.pop() for _ in range(-(-P // BS) + 1)]}
    return reqs

def play_consumer(conn, reqs, seed):
    rng = random.Random(2000 + seed)
    out, seen = [], set()
    R = {rid: NS(request_id=rid, prompt_token_ids=list(range(r["P"])),
                 kv_transfer_params={"transfer_id": r["tid"]} if r["tid"] else None,
                 all_token_ids=list(range(r["P"] + 2))) for rid, r in reqs.items()}
    for rid, r in reqs.items():  # the scheduler asks, then allocates
        m = conn.get_num_new_matched_tokens(R[rid], r["pre"])
        out.append(("matched", rid, m))
        conn.update_state_after_alloc(R[rid], NS(get_block_ids=lambda b=r["blocks"]: (b,)),
                                      m[0] or 0)
    for step in range(6):
        new, cached = [], []
        for rid, r in reqs.items():
            if step < r["start"]:
                continue
            if rid not in seen and r["kind"] == "new":
                new.append(rid); seen.add(rid)
            elif rid not in seen and r["kind"] == "resumed":
                cached.append((rid, rng.randint(0, r["P"]), True)); seen.add(rid)
            elif rid in seen and rng.random() < 0.5:
                cached.append((rid, r["P"] + step, False))  # a decode step
        cached.sort(key=lambda c: not c[2])  # vLLM lists resumed requests first
        so = NS(scheduled_new_reqs=[NS(req_id=rid, prompt_token_ids=R[rid].prompt_token_ids,
                                       block_ids=(reqs[rid]["blocks"],),
                                       num_computed_tokens=reqs[rid]["pre"]) for rid in new],
                num_scheduled_tokens={**{rid: 1 for rid in new}, **{c[0]: 1 for c in cached}},
                scheduled_cached_reqs=NS(req_ids=[c[0] for c in cached],
                                         num_computed_tokens=[c[1] for c in cached],
                                         new_block_ids=[(reqs[c[0]]["blocks"][:2],)
                                                        for c in cached],
                                         resumed_req_ids={c[0] for c in cached if c[2]}))
        out.append(("meta", rows(conn.build_connector_meta(so))))
    for rid in reqs:
        out.append(("finished", rid, conn.request_finished(R[rid], [])))
    return out

n = 0
for seed in range(40):
    reqs, steps = producer_trace(seed)
    a = play_producer(Ours(cfg(True), KVConnectorRole.SCHEDULER), reqs, steps)
    b = play_producer(Ref(cfg(True), KVConnectorRole.SCHEDULER), reqs, steps)
    assert a == b, ("producer", seed, [(x, y) for x, y in zip(a, b) if x != y][:2])
    creqs = consumer_trace(seed)
    a = play_consumer(Ours(cfg(False), KVConnectorRole.SCHEDULER), creqs, seed)
    b = play_consumer(Ref(cfg(False), KVConnectorRole.SCHEDULER), creqs, seed)
    assert a == b, ("consumer", seed, [(x, y) for x, y in zip(a, b) if x != y][:2])
    n += sum(len(x[1]) for x in a if x[0] == "meta")
print("RANDOM SCHEDULER OK", n)
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_scheduler_side_matches_the_reference_on_random_traces(tmp_path):
    """40 seeded random traces per role, played into both connectors'
    scheduler sides: producer chunked prefills of random sizes interleaved
    over steps (some restarted in new blocks after preemption, some without
    a transfer id), consumer requests with a locally cached prefix, requests
    first seen resumed, and decode steps.  Matched tokens, request metadata
    and finish answers must be identical at every step."""
    pytest.importorskip("vllm")
    code = SCHED_RANDOM.replace("ROOT", repr(ROOT)).replace("REF", repr(REF))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=900, cwd=str(tmp_path))
    assert out.returncode == 0 and "RANDOM SCHEDULER OK" in out.stdout, \
        (out.stdout[-1500:] + out.stderr[-3000:])


QUANT_RANDOM = r"""
import random, sys, types
sys.path.insert(0, ROOT)
sys.path.insert(0, REF)
import torch
from kvserve_hpdps_b200.compression.quantizer import KVServeQuantizer as OQ
from kvserve_v1.compression.quantizer.kvserve_quantizer import KVServeQuantizer as RQ

def same(a, b):
    if torch.is_tensor(a):
        return torch.is_tensor(b) and a.shape == b.shape and a.dtype == b.dtype and torch.equal(a, b)
    if isinstance(a, dict):
        return isinstance(b, dict) and a.keys() == b.keys() and all(same(a[k], b[k]) for k in a)
    if isinstance(a, (list, tuple)):
        return isinstance(b, (list, tuple)) and len(a) == len(b) and all(map(same, a, b))
    return a == b

rng = random.Random(11)
g = torch.Generator().manual_seed(11)
models = {"Qwen2.5-7B-Instruct": (28, 4), "Llama-3.1-8B-Instruct": (32, 8),
          "Qwen2.5-32B-Instruct": (64, 8)}
n = 0
for case in range(60):
    model = rng.choice(sorted(models))
    layers, heads = models[model]
    tp = rng.choice([t for t in (1, 2, 4) if heads % t == 0])
    rank = rng.randrange(tp)
    hk, hv = rng.randint(2, 254), rng.randint(2, 254)
    kw = dict(model_name=model, hybrid_ratio=rng.choice([0.0, 0.1, 0.3, 0.5, 0.8, 1.0,
                                                         rng.random()]),
              high_key_max_value=hk, high_value_max_value=hv,
              low_key_max_value=rng.randint(2, hk), low_value_max_value=rng.randint(2, hv),
              axis_key=rng.choice(["channel", "token", "tensor"]),
              axis_value=rng.choice(["channel", "token", "tensor"]),
              split_type=rng.choice(["head", "layer"]))
    if tp > 1:
        kw.update(tensor_parallel_size=tp, tp_rank=rank)
    oq, rq = OQ(**kw), RQ(**kw)
    dtype = rng.choice([torch.bfloat16, torch.float16])
    for _ in range(2):
        layer = rng.randrange(layers)
        shape = (2, rng.randint(1, 6), rng.choice([1, 16]), heads // tp, 128)
        x = torch.randn(shape, generator=g) * rng.choice([0.1, 1.0, 20.0])
        x[..., rng.randrange(128)] *= 12  # an outlier channel
        x = x.to(dtype)
        qo, mo = oq.quantize(layer, x)
        qr, mr = rq.quantize(layer, x)
        assert torch.equal(qo, qr) and same(mo, mr), ("quantize", case, kw, shape, layer)
        do, dr = oq.dequantize(layer, qo, mo), rq.dequantize(layer, qr, mr)
        assert same(do, dr), ("dequantize", case, kw, shape, layer)
        n += 1
print("QUANT RANDOM OK", n)
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_quantizer_matches_the_reference_on_random_configs(tmp_path):
    """60 seeded random quantizer configurations (model head-score table,
    hybrid ratio, the four level counts, key/value axes, head or layer
    split, TP size and rank) on random bf16/fp16 KV with an outlier channel:
    codes, metadata and reconstruction equal the reference's quantizer's."""
    code = QUANT_RANDOM.replace("ROOT", repr(ROOT)).replace("REF", repr(REF))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=900, cwd=str(tmp_path))
    assert out.returncode == 0 and "QUANT RANDOM OK" in out.stdout, \
        (out.stdout[-1500:] + out.stderr[-3000:])


TRANSFORM = r"""
import sys
sys.path.insert(0, ROOT)
sys.path.insert(0, STANDIN)
sys.path.insert(0, REF)
import torch
from kvserve_hpdps_b200.compression.transformer import HadamardTransform as OH
from kvserve_v1.compression.transformer.hadamard_func import HadamardTransform as RH
g = torch.Generator().manual_seed(5)
n = 0
for seed in (0x3333, 0xC0FEBABE):
    o, r = OH(seed), RH(seed)
    for D in (128, 96, 64, 80):          # power-of-two chunks for the others
        for dtype in (torch.float32, torch.bfloat16, torch.float16):
            for layer in (0, 7, 31):
                x = (torch.randn(3, 16, 4, D, generator=g) * 4).to(dtype)
                yo, yr = o.transform(layer, x), r.transform(layer, x)
                assert yo.dtype == yr.dtype == dtype and yo.shape == yr.shape
                tol = {torch.float32: 1e-5, torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10}
                torch.testing.assert_close(yo.float(), yr.float(), rtol=tol[dtype],
                                           atol=tol[dtype] * 4)
                zo, zr = o.inverse(layer, yo), r.inverse(layer, yo)
                torch.testing.assert_close(zo.float(), zr.float(), rtol=tol[dtype],
                                           atol=tol[dtype] * 4)
                if dtype == torch.float32:
                    torch.testing.assert_close(zo, x, rtol=1e-5, atol=1e-5)
                n += 1
print("TRANSFORM OK", n)
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_hadamard_transform_matches_the_reference(tmp_path):
    """The reference's own HadamardTransform (its FWHT extension replaced by
    the plain-PyTorch stand-in of the same function) against ours: forward
    and inverse for two seeds, power-of-two and chunked head sizes, fp32 /
    bf16 / fp16, several layers -- equal within one rounding of the dtype
    (the FWHT's fp32 summation order may differ); the fp32 round trip
    returns the input."""
    code = TRANSFORM.replace("ROOT", repr(ROOT)).replace("REF", repr(REF)).replace(
        "STANDIN", repr(os.path.join(ROOT, "baseline", "standin")))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd=str(tmp_path))
    assert out.returncode == 0 and "TRANSFORM OK" in out.stdout, \
        (out.stdout[-1500:] + out.stderr[-3000:])


TRANSFORM_WIRE = r"""
import sys
sys.path.insert(0, ROOT)
sys.path.insert(0, STANDIN)
sys.path.insert(0, REF)
import torch
from kvserve_hpdps_b200.compression import wire as OW
from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter as Ours
from kvserve_v1.compression import wire as RW
from kvserve_v1.compression.manager import KVCompressionAdapter as Ref
L, T, H, D = 4, 256, 4, 128
g = torch.Generator().manual_seed(3)
x = torch.randn((L, 2, 1, T, H, D), generator=g)
x[:, 0, ..., :4] *= 12
x = x.to(torch.bfloat16)
qc = {"model_name": "Qwen2.5-7B-Instruct", "hybrid_ratio": 0.3, "high_key_max_value": 16,
      "high_value_max_value": 16, "low_key_max_value": 12, "low_value_max_value": 16,
      "axis_key": "channel", "axis_value": "token", "split_type": "head"}
spec = {"enabled": True, "pipeline": ["transformer", "quantizer"],
        "transformer_config": {"transform_type": "hadamard", "seed": 0x3333},
        "quantizer_config": qc, "min_compress_size": 0}
ours = Ours(dict(spec, backend="generic"), H, D, model_name="Qwen2.5-7B-Instruct", num_layers=28)
ref = Ref(spec, H, D, model_name="Qwen2.5-7B-Instruct")
def close(a, b, what):
    a, b = a.float().reshape(-1), b.float().reshape(-1)
    err = (a - b).abs().max().item()
    assert err <= 0.02 * b.abs().max().item(), (what, err)
cd, rc = ours.compress(x, "a"), ref.compress(x, "b")
co, cr = cd.compressed_tensor.view(torch.uint8).reshape(-1), rc.compressed_tensor.view(
    torch.uint8).reshape(-1)
assert co.shape == cr.shape and (co == cr).float().mean().item() > 0.999, "codes"
w = OW.build_wire(cd, 512 << 20)
by_ref = ref.decompress(RW.restore_from_wire(RW.CompressedWire(w.meta, w.body_chunks,
                                                               w.aux_tensors)))
close(by_ref, ours.decompress(cd), "ours -> reference")
rw = RW.build_wire(rc, 512 << 20)
by_ours = ours.decompress(OW.restore_from_wire(OW.CompressedWire(rw.meta, rw.body_chunks,
                                                                 rw.aux_tensors)))
close(by_ours, ref.decompress(rc), "reference -> ours")
cos = torch.nn.functional.cosine_similarity(by_ours.float().reshape(-1), x.float().reshape(-1), 0)
assert cos.item() > 0.98, cos
print("TRANSFORM WIRE OK", (co == cr).float().mean().item())
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_transform_pipeline_messages_cross_between_the_frameworks(tmp_path):
    """Transformer + quantizer pipeline messages (the reference's Hadamard
    with the FWHT stand-in): the code bodies agree byte for byte except where
    the two FWHT summation orders round a value onto the other side of a
    quantization step (under 0.1 % of the bytes), and each framework decodes
    the other's message to the other's own reconstruction."""
    code = TRANSFORM_WIRE.replace("ROOT", repr(ROOT)).replace("REF", repr(REF)).replace(
        "STANDIN", repr(os.path.join(ROOT, "baseline", "standin")))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd=str(tmp_path))
    assert out.returncode == 0 and "TRANSFORM WIRE OK" in out.stdout, \
        (out.stdout[-1500:] + out.stderr[-3000:])


CTL_RANDOM = r"""
import random, sys
sys.path.insert(0, ROOT)
sys.path.insert(0, REF)
from kvserve_hpdps_b200.controller.analytical_model import AnalyticalModel
from kvserve_hpdps_b200.controller.online_controller import OnlineController as Ours
from kvserve_hpdps_b200.controller.profile_library import ProfileLibrary as OursLib
from kvserve_hpdps_b200.offline.library_export import build_library, write_library
from kvserve_hpdps_b200.offline.search_space import Candidate
from kvserve_v1.compression.controller.online_controller import OnlineController as Ref
from kvserve_v1.compression.controller.profile_library import ProfileLibrary as RefLib
rng = random.Random(3)
n = 0
for lib_i in range(25):
    evals = []
    for _ in range(rng.randint(1, 9)):
        hk, hv = rng.choice([16, 12, 8]), rng.choice([16, 12, 8])
        c = Candidate(rng.choice([0.0, 0.3, 0.5, 0.8, 1.0]), hk, hv,
                      rng.choice([x for x in (12, 8, 6, 4) if x <= hk]),
                      rng.choice([x for x in (8, 6, 4) if x <= hv]))
        evals.append({"candidate": c.key() + f"_{len(evals)}", "config": c.quantizer_config(),
                      "accuracy": rng.uniform(0.85, 1.0), "compression_ratio": rng.uniform(1.5, 12),
                      "harmonic_speed_mbps": rng.uniform(500, 200000)})
    edges = sorted(rng.sample([0.8, 0.85, 0.9, 0.93, 0.95, 0.97, 0.99], rng.randint(2, 5)))
    bws = sorted(rng.sample([10, 100, 1000, 5000, 20000, 100000, 1000000], rng.randint(2, 6)))
    path = TMP + f"/lib{lib_i}.json"
    write_library(path, build_library(evals, "m", acc_edges=edges + [1.0001],
                                      bw_edges_mbps=bws, k=rng.randint(1, 4)))
    ours = Ours(OursLib(path), epsilon=0.0, model=AnalyticalModel(reference_transfer_term=True))
    ref = Ref(RefLib(path), epsilon=0.0)
    for _ in range(60):
        V = rng.choice([1e6, 64e6, 470e6, 4e9])
        B = 10 ** rng.uniform(0, 6.5)
        slo = rng.choice([1.0, 20.0, 200.0, 2000.0, 1e9])
        acc = rng.uniform(0.8, 1.0)
        tm = rng.choice([0.0, 10.0, 100.0])
        po, co = ours.select_profile(V, B, tm, slo, acc)
        pr, cr_ = ref.select_profile(V, B, tm, slo, acc)
        ido = None if po is None else po.profile_id
        idr = None if pr is None else pr.profile_id
        assert ido == idr, (lib_i, V, B, slo, acc, ido, idr, co, cr_)
        for k in ("bucket_id", "interval_id", "action", "num_candidates", "T_hat", "T_eff"):
            if k in cr_:
                a, b = co.get(k), cr_[k]
                assert a == b or (isinstance(b, float) and abs(a - b) <= 1e-9 * max(1, abs(b))), \
                    (lib_i, k, co, cr_)
        if po is not None:
            t = rng.uniform(1, 500)
            ours.update(co, t)
            ref.update(cr_, t)
        n += 1
    so, sr = ours.get_statistics(), ref.get_statistics()
    for k in ("total_decisions", "exploit_count", "explore_count", "no_compression_count"):
        assert so[k] == sr[k], (lib_i, k, so, sr)
print("RANDOM CONTROLLER OK", n)
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_controller_decisions_match_the_reference_on_random_libraries(tmp_path):
    """25 random profile libraries (random profiles, accuracy buckets,
    bandwidth intervals and candidate counts), 60 random requests each
    (volume, bandwidth, model time, SLO, accuracy requirement), with bandit
    updates in between: both controllers pick the same profile with the same
    context and keep the same statistics."""
    code = CTL_RANDOM.replace("ROOT", repr(ROOT)).replace("REF", repr(REF)) \
        .replace("TMP", repr(str(tmp_path)))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd=str(tmp_path))
    assert out.returncode == 0 and "RANDOM CONTROLLER OK" in out.stdout, \
        (out.stdout[-1500:] + out.stderr[-3000:])


OFFLINE = r"""
import sys, types
sys.path.insert(0, ROOT)
sys.path.insert(0, REF)
# the reference's offline caches were written for transformers 4.x
# (CacheConfig) and import its FWHT extension; only pure functions run here
import transformers.cache_utils as cu
if not hasattr(cu, "CacheConfig"):
    class CacheConfig:
        def __init__(self, *a, **k):
            pass
    cu.CacheConfig = CacheConfig
sys.modules.setdefault("fast_hadamard_transform", types.ModuleType("fast_hadamard_transform"))
import torch
from kvserve_hpdps_b200.offline import caches as C
from kvserve_hpdps_b200.offline.caches.common import minmax_codes, minmax_values
from kvserve_v1.offline_search.src.cache import cache_utils as RU
from kvserve_v1.offline_search.src.cache import cachegen_utils as RC
from kvserve_v1.offline_search.src.cache import duoattn_utils as RD
for L in (4, 28, 32, 64):
    for lvl in (1, 2, 3):
        r = RC.CacheGenCacheConfig(model_layers=L, quantization_level=lvl)
        ns = types.SimpleNamespace(**{k: getattr(r, k) for k in (
            "model_layers", "quantization_level", "high_max_value", "mid_max_value",
            "low_max_value")})
        assert RC.CacheGenCache.make_quantized_bins(ns) == C.cachegen_bins(
            C.CacheGenCacheConfig(model_layers=L, quantization_level=lvl)), ("bins", L, lvl)
g = torch.Generator().manual_seed(0)
x = torch.randn(3, 50, 16, generator=g) + 2.0
assert torch.equal(RD.search_hyperplane(x.clone()), C.search_hyperplane(x.clone())), "hyperplane"
for dtype in (torch.bfloat16, torch.float16, torch.float32):
    kv = (torch.randn(1, 4, 97, 128, generator=g) * 3).to(dtype)
    for maxv in (4, 12, 16, 255):
        for axis in ([2], [1, 3], [-1], [0, 1, 2, 3]):
            qr, mr = RU.CustomCache._quantize(None, maxv, kv, axis)
            qo, mo = minmax_codes(kv, maxv, axis)
            assert torch.equal(qr, qo) and torch.equal(mr, mo), ("quantize", dtype, maxv, axis)
            assert torch.equal(RU.CustomCache._dequantize(None, qr, mr),
                               minmax_values(qo, mo)), ("dequantize", dtype, maxv, axis)
    empty = kv[:, :0]
    qr, mr = RU.CustomCache._quantize(None, 12, empty, [2])
    qo, mo = minmax_codes(empty, 12, [2])
    assert qr.shape == qo.shape and mr.shape == mo.shape, "empty"
# affine transforms from one parameter file in the reference's format
import os, tempfile
from kvserve_hpdps_b200.offline.caches.transforms import AffineTransform as OA
D = 128
for mode in ("diag", "full"):
    params = {}
    for layer in range(2):
        sd = {"clip_k": torch.randn(D, generator=g) + 3, "clip_v": torch.randn(D, generator=g) + 3}
        if mode == "diag":
            sd["log_scale"] = torch.randn(D, generator=g) * 2
        else:
            sd["linear.weight"] = torch.eye(D) + 0.05 * torch.randn(D, D, generator=g)
        params[layer] = {"state_dict": sd}
    path = os.path.join(tempfile.mkdtemp(), "affine.pt")
    torch.save(params, path)
    ra = RU.AffineTransform(D, mode=mode, params_path=path, device="cpu")
    oa = OA(D, mode=mode, params_path=path)
    for dtype in (torch.float32, torch.bfloat16):
        x = (torch.randn(1, 4, 33, D, generator=g) * 4).to(dtype)
        for layer in (0, 1, 5):  # layer 5: default parameters on both sides
            for kind in ("k", "v"):
                yr, yo = ra.transform(x, layer, kind), oa.transform(x, layer, kind)
                assert torch.equal(yr, yo), ("affine", mode, dtype, layer, kind)
                assert torch.equal(ra.inverse(yr, layer), oa.inverse(yo, layer)), \
                    ("affine inverse", mode, dtype, layer)
        assert torch.equal(oa.forward_transform(x, "v", 1), oa.transform(x, 1, "v"))
print("OFFLINE OK")
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_offline_cache_math_matches_the_reference(tmp_path):
    """Pure pieces of the reference's offline caches against ours: CacheGen's
    per-layer bins, DuoAttention's streaming-head hyperplane, and the custom
    cache's min-max quantize/dequantize over every axis choice and dtype."""
    code = OFFLINE.replace("ROOT", repr(ROOT)).replace("REF", repr(REF))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd=str(tmp_path))
    assert out.returncode == 0 and "OFFLINE OK" in out.stdout, \
        (out.stdout[-1500:] + out.stderr[-3000:])
