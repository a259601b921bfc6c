"""Benchmark drivers on CPU: argument handling of ``bench.py`` and the
size/step planning and report of the handoff sweep (the timed runs need
GPUs)."""

import importlib.util
import os

import pytest

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _sweep():
    spec = importlib.util.spec_from_file_location(
        "handoff_sweep", os.path.join(ROOT, "examples", "handoff_sweep.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_bench_modes_and_labels():
    a = bench.parse_args([])
    assert a.compression == "default" and bench.hybrid_ratio(a) == 0.8
    # the headline runs the stage set both arms can run: byte codes, no entropy coder
    assert a.codec == "none"
    assert bench.compression_label(a) == \
        "default mode: Hadamard + hybrid 0.8 12/8/6/4, u8 codes, no entropy codec"
    assert bench.compression_label(a, "rans").endswith("4-bit codes + rANS")
    a = bench.parse_args(["--hybrid-ratio", "0.3", "--codec", "bitpack"])
    assert bench.quant_config(a)["quantizer_config"]["hybrid_ratio"] == 0.3
    assert "bit-packed" in bench.compression_label(a)
    assert bench.compression_label(bench.parse_args(["--compression", "off"])) == \
        "off (raw bf16 blocks)"


def test_bench_line_config_is_the_same_for_both_arms():
    """The driver compares the two arms' ``config``: it must not depend on
    the arm; arm-specific descriptions sit outside it."""
    ours = bench.parse_args([])
    ref = bench.parse_args(["--impl", "reference"])
    res = {"ms": 80.0, "cr": 1.97, "pairs": 1, "launches": 100, "pipeline": "p",
           "transport": "local"}
    a = bench.build_line(ours, dict(res), 1)
    b = bench.build_line(ref, dict(res), 1)
    assert a["config"] == b["config"]
    assert a["impl"] == "ours" and b["impl"] == "reference"
    assert a["value"] == 80.0 / (20 * 8)
    # N >= 2: value is per pair (weak scaling), aggregate throughput is separate
    c = bench.build_line(bench.parse_args(["--gpus", "8"]), dict(res, pairs=4), 8)
    assert c["value"] == a["value"] and c["config"]["global_batch"] == 32
    assert abs(c["aggregate_gbps"] - 4 * a["aggregate_gbps"]) < 1.0


def test_sweep_plan_and_report():
    sw = _sweep()
    assert sw.BYTES_PER_TOKEN == 57344
    assert sw.DEFAULT_TOKENS[0] * sw.BYTES_PER_TOKEN < 1.1e6
    assert sw.DEFAULT_TOKENS[-1] * sw.BYTES_PER_TOKEN > 4 * 2 ** 30
    assert sw.steps_for(16) == 40 and sw.steps_for(74912) == 3
    a = sw.point_args(bench, 2, 4096, "h0.3", 3)
    assert (a.tokens, a.requests_per_step, a.compression, a.hybrid_ratio, a.no_e2e) == \
        (4096, 1, "default", 0.3, True)
    assert sw.point_args(bench, 1, 16, "off", 3).compression == "off"
    rows = [{"impl": "ours", "tokens": 16, "mode": "off", "ms_per_request": 0.01,
             "raw_gbps": 91.0, "compression_ratio": 1.0},
            {"impl": "reference", "tokens": 16, "mode": "off", "ms_per_request": 0.05,
             "raw_gbps": 18.0, "compression_ratio": 1.0},
            {"impl": "reference", "unavailable": "x"}]
    table = sw.render(rows)
    assert "| 0.9 | off | 0.01 | 91.0 | 1.0 | 0.05 | 18.0 | 1.0 | 5.0x |" in table


def test_copy_grids_scale_with_segment_size():
    from kvserve_hpdps_b200.ops import kernels as K
    assert K._grid_per_seg([(0, 0, 1000)], 16) == 16
    assert K._grid_per_seg([(0, 0, 64 << 20), (0, 0, 100)], 16) == 256
    assert K._grid_per_seg([(0, 0, 4 << 30)], 32) == 1184


def test_ttft_harness_prompts_are_deterministic():
    """Both sides of a cross-node run generate the same requests."""
    spec = importlib.util.spec_from_file_location(
        "pd_ttft", os.path.join(ROOT, "examples", "pd_ttft.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    a, b = mod.prompts(4, 64), mod.prompts(4, 64)
    assert a == b and len(a) == 4 and all(len(p) == 64 for p in a)
    assert all(0 <= t < mod.QWEN25_7B["vocab_size"] for p in a for t in p)


def test_rank_pairing_for_every_scaling_point():
    """N = 1, 2, 4, 8: rank r < N/2 produces for consumer r + N/2, both with
    the same pair id; N = 1 runs both roles; odd N is rejected."""
    import bench
    assert bench._roles(1, 0) == ("both", 1)
    for world in (2, 4, 8):
        pairs = world // 2
        roles = [bench._roles(world, r) for r in range(world)]
        assert all(p == pairs for _, p in roles)
        assert [r for r, _ in roles] == ["producer"] * pairs + ["consumer"] * pairs
        for r in range(pairs):
            assert r % pairs == (r + pairs) % pairs  # the pair id both sides derive
    with pytest.raises(SystemExit):
        bench._roles(3, 0)


def test_reference_arm_imports_nothing_of_this_package():
    """The reference arm's workload, labels and pipeline set-up come from
    bench.py itself: running them in a fresh interpreter loads no module of
    this package."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r); import bench; "
            "a = bench.parse_args(['--impl', 'reference']); "
            "bench.compression_label(a); bench.hybrid_ratio(a); "
            "bench.outlier_channels(4, 128, 0.03, 3); "
            "print(sorted(m for m in sys.modules if m.startswith('kvserve_hpdps_b200')))" % ROOT)
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip().splitlines()[-1] == "[]"


def test_reference_e2e_loop_and_its_failure_path(monkeypatch):
    """The reference arm's end-to-end loop: the same steps plus a 4-byte
    result read per step, value per request; a failing step gives an
    ``unavailable`` entry instead of breaking the line (CPU stand-ins for
    events, synchronisation and pinned memory)."""
    import torch

    class Ev:
        t = 0.0

        def record(self):
            Ev.t += 5.0
            self.at = Ev.t

        def elapsed_time(self, other):
            return other.at - self.at

    monkeypatch.setattr(bench, "_events", lambda: (Ev(), Ev()))
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    real_empty = torch.empty
    monkeypatch.setattr(torch, "empty", lambda *a, pin_memory=False, **k: real_empty(*a, **k))
    args = bench.parse_args(["--impl", "reference", "--steps", "3", "--requests-per-step", "2"])
    cache = torch.arange(2 * 4 * 16 * 2 * 8, dtype=torch.float32).to(torch.bfloat16).view(
        2, 4, 16, 2, 8)
    seen = []
    e2e = bench._ref_e2e(args, 1, "cpu", seen.append, 7, cache, [3, 1], 1234, 1)
    assert seen == [7, 8, 9] and e2e["steps"] == 3
    assert e2e["value"] == round(5.0 / (3 * 2), 5) and e2e["unit"] == "ms/request"
    assert e2e["h2d_bytes_per_step"] == 1234 and e2e["d2h_bytes_per_step"] == 4

    def bad(s):
        raise RuntimeError("boom")
    out = bench._ref_e2e(args, 1, "cpu", bad, 0, cache, [0], 1, 1)
    assert out == {"unavailable": "RuntimeError: boom"}
    line = bench.build_line(args, {"ms": 30.0, "cr": 2.0, "pairs": 1, "pipeline": "p",
                                   "transport": "local", "e2e": e2e}, 1)
    assert line["impl"] == "reference" and line["e2e"] == e2e


def test_environment_check_report_and_exit_code():
    """``python -m kvserve_hpdps_b200``: versions, native library, GPUs; the
    exit code says whether the fused path can run on every visible GPU."""
    from kvserve_hpdps_b200 import __main__ as env
    rep = env.report()
    assert rep["package"] and rep["native"]["loaded"] is True and rep["gpus"] == []
    assert rep["native"]["cpu_codec_ok"] is True
    assert env.exit_code(rep) == 2  # no GPU here
    b200 = {"index": 0, "name": "B200", "capability": "10.0", "fused_path": True}
    h100 = dict(b200, capability="9.0", fused_path=False)
    assert env.exit_code(dict(rep, gpus=[b200])) == 0
    assert env.exit_code(dict(rep, gpus=[b200, h100])) == 1
    assert env.exit_code(dict(rep, gpus=[b200], native={"loaded": False})) == 1


def test_roofline_terms_of_each_path(monkeypatch):
    """Algorithmic bytes per 470 MB request: two reads of the input, the
    codes (or the rANS stream) written into the consumer's memory and read,
    the rANS codes' round trip on each side, the bf16 output."""
    monkeypatch.setattr(bench, "_peaks", lambda: (6452.5, "measured"))
    a = bench.parse_args([])
    raw = 28 * 2 * 8192 * 4 * 128 * 2
    r1 = bench.roofline(a, 1, "none", 1.988, 0.587)
    assert r1["limited_by"] == "hbm"
    assert abs(r1["bound_ms"] - 4 * raw / 6452.5e6) < 1e-4 and r1["fraction"] == 0.496
    r2 = bench.roofline(a, 2, "none", 1.988, 0.479)
    assert r2["limited_by"] == "nvlink" and abs(r2["bound_ms"] - raw / 2 / 770e6) < 1e-4
    r3 = bench.roofline(a, 2, "rans", 9.18, 0.585)
    assert r3["limited_by"] == "hbm-producer"
    assert abs(r3["terms_ms"]["hbm-producer"] - (2 * raw + raw / 2) / 6452.5e6) < 1e-4
    assert abs(r3["terms_ms"]["nvlink"] - raw / 9.18 / 770e6) < 1e-4
    line = bench.build_line(bench.parse_args(["--impl", "reference"]),
                            {"ms": 8 * 20 * 28.06, "cr": 1.988, "pairs": 1, "pipeline": "p",
                             "transport": "local"}, 1)
    assert line["roofline"]["fraction"] < 0.02  # the same bound for the reference arm


def test_full_path_summary_carries_its_roofline():
    from types import SimpleNamespace
    a = bench.parse_args([])
    wl = SimpleNamespace(B=8, bf16_bytes_per_request=28 * 2 * 8192 * 4 * 128 * 2)
    res = {"ms": 20 * 8 * 0.89, "launches": 220, "wire_bytes_per_step":
           wl.bf16_bytes_per_request * 8 / 9.18, "e2e": {"value": 0.915}}
    out = bench._summary(a, wl, res, 1, "rans")
    assert out["compression_ratio"] == 9.18 and out["e2e"] == {"value": 0.915}
    assert out["roofline"]["limited_by"] == "hbm" and 0.2 < out["roofline"]["fraction"] < 0.5


def test_every_package_module_imports():
    """Each module of the package imports on a CPU-only machine (the native
    library's own file is not a Python module)."""
    import importlib
    import pkgutil

    import kvserve_hpdps_b200 as pkg
    bad = []
    for m in pkgutil.walk_packages(pkg.__path__, pkg.__name__ + "."):
        if m.name.endswith(".libkvs_b200") or ".compat.kvserve_v1" in m.name:
            continue
        try:
            importlib.import_module(m.name)
        except Exception as e:  # noqa: BLE001
            bad.append((m.name, repr(e)[:200]))
    assert not bad, bad
