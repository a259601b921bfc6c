"""Controller: profile library lookups, analytical model, bandit state and
the two-tier selection (CPU only)."""

import json

import pytest

from kvserve_hpdps_b200.controller import (AnalyticalModel, BanditStateManager, OnlineController,
                                           Profile, ProfileLibrary)


def _profile(pid, cr, speed, acc, hr=0.3):
    return {"profile_id": pid, "metadata": {"hybrid_ratio": hr},
            "compression_config": {"enabled": True, "pipeline": ["quantizer", "codec"],
                                   "quantizer_config": {"hybrid_ratio": hr}},
            "performance_metrics": {"compression_ratio": cr, "harmonic_speed_mbps": speed},
            "quality_metrics": {"accuracy": acc}}


def library_dict():
    profiles = [_profile("p_light", 3.0, 200000.0, 0.99, 0.0),
                _profile("p_mid", 6.0, 100000.0, 0.95, 0.3),
                _profile("p_heavy", 9.0, 50000.0, 0.93, 1.0)]
    return {"library_metadata": {"model_name": "Qwen2.5-7B-Instruct", "dataset": "synthetic"},
            "accuracy_buckets": [
                {"bucket_id": 0, "acc_range": [0.9, 0.95], "pareto_profiles": profiles,
                 "bandwidth_intervals": [
                     {"interval_id": 0, "x_range": [0.0, 1e-4],
                      "candidate_profile_ids": ["p_light", "p_mid"]},
                     {"interval_id": 1, "x_range": [1e-4, 1.0],
                      "candidate_profile_ids": ["p_mid", "p_heavy"],
                      "model_optimal_profile_id": "p_heavy"}]},
                {"bucket_id": 1, "acc_range": [0.95, 1.01], "pareto_profiles": profiles[:1],
                 "bandwidth_intervals": [{"interval_id": 0, "x_range": [0.0, 1.0],
                                          "candidate_profile_ids": ["p_light"]}]}]}


@pytest.fixture
def lib_path(tmp_path):
    p = tmp_path / "lib.json"
    p.write_text(json.dumps(library_dict()))
    return str(p)


def test_library_lookups(lib_path):
    lib = ProfileLibrary(lib_path)
    assert lib.get_num_profiles() == 3 and lib.get_num_buckets() == 2
    assert lib.find_bucket(0.92)["bucket_id"] == 0
    assert lib.find_bucket(0.99)["bucket_id"] == 1
    assert lib.find_bucket(0.5)["bucket_id"] == 0  # closest bucket
    b = lib.find_bucket(0.92)
    assert lib.find_interval(b, 50000.0)["interval_id"] == 0   # 1/B = 2e-5
    assert lib.find_interval(b, 1000.0)["interval_id"] == 1    # 1/B = 1e-3
    assert lib.find_interval(b, 0.5)["interval_id"] == 1       # past the last -> last
    assert lib.get_optimal_profile(b, b["bandwidth_intervals"][1]).profile_id == "p_heavy"
    with pytest.raises(FileNotFoundError):
        ProfileLibrary("/nonexistent.json")
    with pytest.raises(ValueError):
        ProfileLibrary(data={"accuracy_buckets": []})


def test_profile_properties():
    p = Profile.from_dict(_profile("x", 4.0, 1000.0, 0.9))
    assert p.critical_bandwidth == pytest.approx(750.0)
    assert Profile.from_dict(p.to_dict()) == p


def test_analytical_model():
    p = Profile.from_dict(_profile("x", 4.0, 1000.0, 0.9))
    m = AnalyticalModel()
    V = 100 * 1024 * 1024  # 100 MB
    assert m.predict_latency(p, V, 100.0, 5.0) == pytest.approx(5 + 100.0 + 250.0)
    assert m.predict_baseline_latency(V, 100.0, 5.0) == pytest.approx(1005.0)
    assert m.check_benefit(p, 700.0) and not m.check_benefit(p, 800.0)
    ref = AnalyticalModel(reference_transfer_term=True)
    assert ref.predict_latency(p, V, 100.0, 0.0) == pytest.approx(100.0 + 4000.0)


def test_bandit_ewma_and_persistence(tmp_path):
    b = BanditStateManager(alpha=0.5)
    b.update(0, 1, "p_a_b", 10.0)
    b.update(0, 1, "p_a_b", 20.0)
    assert b.get_stats(0, 1, "p_a_b") == (2, pytest.approx(12.5))
    path = str(tmp_path / "s" / "bandit.json")
    b.save(path)
    c = BanditStateManager()
    c.load(path)
    assert c.alpha == 0.5 and c.get_stats(0, 1, "p_a_b") == (2, pytest.approx(12.5))
    assert "0_1_p_a_b" in json.load(open(path))["state"]


def test_controller_selects_and_learns(lib_path):
    ctl = OnlineController(ProfileLibrary(lib_path), epsilon=0.0, seed=1)
    V = 470 * 1024 * 1024
    prof, ctx = ctl.select_profile(V, 1000.0, 0.0, float("inf"), 0.92)
    assert prof is not None and ctx["action"] == "exploit"
    assert prof.profile_id == "p_heavy"  # slow link: strongest compression
    prof2, _ = ctl.select_profile(V, 60000.0, 0.0, float("inf"), 0.92)
    assert prof2.profile_id in ("p_light", "p_mid")
    # a residual that makes p_heavy look slow flips the exploit choice
    for _ in range(20):
        ctl.update(ctx, ctx["T_hat"] + 1e6)
    prof3, _ = ctl.select_profile(V, 1000.0, 0.0, float("inf"), 0.92)
    assert prof3.profile_id == "p_mid"
    st = ctl.get_statistics()
    assert st["total_decisions"] == 3 and st["bandit_states"] == 1


def test_controller_no_compression_reasons(lib_path):
    ctl = OnlineController(ProfileLibrary(lib_path), epsilon=0.0)
    prof, ctx = ctl.select_profile(1e9, 1e9, 0.0, float("inf"), 0.92)
    assert prof is None and ctx["reason"] == "no_benefit"
    prof, ctx = ctl.select_profile(1e9, 1000.0, 0.0, 1.0, 0.92)
    assert prof is None and ctx["reason"] == "slo_violation"
    assert ctl.get_statistics()["no_compression_count"] == 2


def test_controller_exploration_is_seeded(lib_path):
    picks = []
    for _ in range(2):
        ctl = OnlineController(ProfileLibrary(lib_path), epsilon=1.0, seed=7)
        picks.append([ctl.select_profile(1e8, 1000.0, 0.0, float("inf"), 0.92)[0].profile_id
                      for _ in range(10)])
    assert picks[0] == picks[1]
    assert set(picks[0]) <= {"p_mid", "p_heavy"}
