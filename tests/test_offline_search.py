"""Offline search: space, dominance pruning, BO on a synthetic objective,
KV evaluator on CPU (generic pipeline), library export loaded by the
controller."""

import json
import math
import os

import pytest
import torch

from kvserve_hpdps_b200.offline.bo import ConstraintAwareBO, predicted_cr
from kvserve_hpdps_b200.offline.library_export import build_library, write_library
from kvserve_hpdps_b200.offline.search_space import (Candidate, enumerate_space, is_valid,
                                                     prune_after)


def test_space_valid_and_pruning():
    space = enumerate_space()
    assert space and all(is_valid(c) for c in space)
    assert all(c.low_key_max_value <= c.high_key_max_value for c in space)
    mid = Candidate(0.5, 12, 12, 8, 6)
    # infeasible: everything with no more precision goes
    rest = prune_after(mid, False, space)
    assert mid not in rest
    assert Candidate(0.8, 12, 12, 6, 4) not in rest
    assert Candidate(0.3, 16, 16, 8, 6) in rest
    # feasible: everything with at least as much precision goes
    rest = prune_after(mid, True, space)
    assert Candidate(0.3, 16, 16, 8, 6) not in rest
    assert Candidate(0.8, 12, 12, 6, 4) in rest


def _objective(c: Candidate) -> dict:
    """Accuracy falls with fewer bits; CR rises."""
    cr = predicted_cr(c)
    acc = 1.0 - 0.004 * (cr - 4.0) ** 2 / 4.0
    return {"accuracy": acc, "compression_ratio": cr}


def test_bo_finds_best_feasible():
    space = enumerate_space()
    thr = 0.97
    truth = max((predicted_cr(c) for c in space if _objective(c)["accuracy"] >= thr))
    bo = ConstraintAwareBO(space, _objective, thr, budget=25, patience=8)
    res = bo.run()
    assert res["best"] is not None
    assert res["best"]["accuracy"] >= thr
    assert res["evaluations"] <= 25
    # within 10% of the best feasible CR of the whole space
    assert res["best"]["compression_ratio"] >= 0.9 * truth


def test_kv_evaluator_cpu_and_export(tmp_path):
    from kvserve_hpdps_b200.controller.profile_library import ProfileLibrary
    from kvserve_hpdps_b200.offline.search import run_search
    kv = torch.stack([torch.randn(2, 64, 4, 128) for _ in range(2)], 0)
    res = run_search(kv, "Qwen2.5-7B-Instruct", 5.0, str(tmp_path), budget=4,
                     space={"hybrid_ratio": [0.0, 1.0], "high_key_max_value": [16],
                            "high_value_max_value": [16], "low_key_max_value": [8, 4],
                            "low_value_max_value": [4]},
                     measure_speed=False)
    assert res["evaluations"] >= 2
    for h in res["history"]:
        assert h["compression_ratio"] > 1.5
        assert 0.5 < h["accuracy"] <= 1.0 + 1e-6
    files = os.listdir(tmp_path)
    assert "tolerance_5_results.json" in files and "cr_cache.csv" in files
    lib = ProfileLibrary(str(tmp_path / "profile_library.json"))
    assert lib.get_num_profiles() >= 1
    # resumable: a second run re-uses the cached rows
    res2 = run_search(kv, "Qwen2.5-7B-Instruct", 5.0, str(tmp_path), budget=4, space={
        "hybrid_ratio": [0.0, 1.0], "high_key_max_value": [16], "high_value_max_value": [16],
        "low_key_max_value": [8, 4], "low_value_max_value": [4]}, measure_speed=False)
    assert [h["candidate"] for h in res2["history"]] == [h["candidate"] for h in res["history"]]
    # another search (here another KV shape) does not resume from this cache
    with pytest.raises(ValueError, match="another search"):
        run_search(kv[:1], "Qwen2.5-7B-Instruct", 5.0, str(tmp_path), budget=2,
                   measure_speed=False)


def test_library_export_selection(tmp_path):
    from kvserve_hpdps_b200.controller.online_controller import OnlineController
    from kvserve_hpdps_b200.controller.profile_library import ProfileLibrary
    evals = []
    for c, acc, cr, s in [(Candidate(0.0, 16, 16, 8, 6), 0.995, 3.5, 40000.0),
                          (Candidate(0.8, 12, 8, 6, 4), 0.97, 6.0, 30000.0),
                          (Candidate(1.0, 8, 8, 4, 4), 0.90, 8.5, 20000.0)]:
        evals.append({"candidate": c.key(), "config": c.quantizer_config(), "accuracy": acc,
                      "compression_ratio": cr, "harmonic_speed_mbps": s})
    lib = build_library(evals, "Qwen2.5-7B-Instruct")
    path = tmp_path / "lib.json"
    write_library(str(path), lib)
    pl = ProfileLibrary(str(path))
    assert pl.get_num_profiles() == 3
    b = pl.find_bucket(0.96)
    ids = {p["profile_id"] for p in b["pareto_profiles"]}
    assert Candidate(1.0, 8, 8, 4, 4).key() not in ids  # below the bucket's floor
    # low bandwidth -> highest CR in the bucket; high bandwidth -> fastest
    low = pl.find_interval(b, 150.0)
    assert pl.get_candidate_profiles(b, low)[0].compression_ratio == 6.0
    ctl = OnlineController(pl, epsilon=0.0, seed=0)
    V = 470e6
    prof, ctx = ctl.select_profile(V, 150.0, 10.0, 1e9, 0.96)
    assert prof is not None and prof.compression_ratio == 6.0, ctx


def test_adapter_controller_mode_end_to_end(tmp_path):
    """Library from the exporter -> adapter in controller mode: the selected
    profile depends on the measured bandwidth, the payload round-trips, the
    bandit learns from the observed latency, and fast links send raw KV."""
    from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter

    def spec(cfg):
        return {"enabled": True, "pipeline": ["transformer", "quantizer", "codec"],
                "transformer_config": {"transform_type": "hadamard", "seed": 0x3333},
                "quantizer_config": dict(cfg), "codec_config": {"codec_type": "rans"},
                "backend": "generic", "min_compress_size": 0}
    evals = []
    for c, acc, cr in [(Candidate(0.0, 16, 16, 8, 6), 0.995, 3.5),
                       (Candidate(0.8, 12, 8, 6, 4), 0.97, 6.0)]:
        evals.append({"candidate": c.key(), "config": c.quantizer_config(), "accuracy": acc,
                      "compression_ratio": cr, "harmonic_speed_mbps": 30000.0})
    path = tmp_path / "lib.json"
    write_library(str(path), build_library(evals, "Qwen2.5-7B-Instruct", spec_builder=spec))
    service = {"bandwidth_mbps": 1e9, "slo_ms": 1e9, "accuracy_requirement": 0.96,
               "t_model_ms": 0.0}
    bw = {"v": 150.0}
    ad = KVCompressionAdapter({"mode": "controller", "library_path": str(path), "epsilon": 0.0,
                               "service_config": service}, 4, 128,
                              model_name="Qwen2.5-7B-Instruct", num_layers=28,
                              bandwidth_fn=lambda: bw["v"])
    g = torch.Generator().manual_seed(0)
    x = torch.randn((2, 2, 64, 4 * 128), generator=g).to(torch.bfloat16)
    cd = ad.compress(x, "r1")
    assert cd is not None
    assert cd.metadata["ctrl_profile_id"] == Candidate(0.8, 12, 8, 6, 4).key()
    out = ad.decompress(cd)
    assert out.shape == x.shape
    cos = torch.nn.functional.cosine_similarity(out.float().flatten(), x.float().flatten(), dim=0)
    assert float(cos) > 0.9
    ad.update_controller("r1", 12.5)
    st = ad.get_controller_stats()
    assert st["total_decisions"] == 1 and st["bandit_states"] == 1
    bw["v"] = 1e9  # a link faster than any profile's codec: send raw KV
    assert ad.compress(x, "r2") is None
