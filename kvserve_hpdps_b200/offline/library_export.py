"""Build the controller's profile-library JSON from evaluated candidates.

The reference has no code path from its search output to the library
(profiles were assembled by hand); this exporter produces the schema the
controller loads (``controller/profile_library.py``):

* accuracy buckets from the given edges; a profile belongs to every bucket
  whose lower edge it meets;
* per bucket, the Pareto set over (compression ratio, harmonic speed,
  accuracy);
* bandwidth intervals in x = 1/B (MB/s)^-1 space from the given bandwidth
  edges; per interval, the candidates with the lowest predicted transfer
  latency V/S + V/(cr*B) at the interval's geometric-mid bandwidth (top
  ``k``), and the best one as ``model_optimal_profile_id``.
"""

from __future__ import annotations

import json
import math
from typing import Iterable, Sequence


def _pareto(profiles: list[dict]) -> list[dict]:
    def key(p):
        return (p["performance_metrics"]["compression_ratio"],
                p["performance_metrics"]["harmonic_speed_mbps"], p["quality_metrics"]["accuracy"])
    out = []
    for p in profiles:
        kp = key(p)
        dominated = any(all(a >= b for a, b in zip(key(q), kp)) and key(q) != kp
                        for q in profiles)
        if not dominated:
            out.append(p)
    return out


def build_library(evals: Iterable[dict], model_name: str, dataset: str = "synthetic",
                  acc_edges: Sequence[float] = (0.8, 0.9, 0.95, 0.99, 1.0001),
                  bw_edges_mbps: Sequence[float] = (100, 1000, 10000, 100000, 1000000),
                  k: int = 3, spec_builder=None) -> dict:
    """``evals``: dicts with ``config`` (quantizer config), ``accuracy``,
    ``compression_ratio`` and ``harmonic_speed_mbps`` (as produced by the
    search).  ``spec_builder(config) -> compression dict`` (default: the
    candidate pipeline [transformer, quantizer, codec])."""
    from kvserve_hpdps_b200.offline.evaluators import candidate_spec
    from kvserve_hpdps_b200.offline.search_space import Candidate
    profiles = []
    for e in evals:
        cfg = dict(e["config"])
        cfg.pop("model_name", None)
        spec = spec_builder(cfg) if spec_builder else candidate_spec(Candidate(**cfg), model_name)
        S = e.get("harmonic_speed_mbps") or 1e6
        profiles.append({
            "profile_id": e.get("candidate") or Candidate(**cfg).key(),
            "metadata": {"model_name": model_name, "dataset": dataset},
            "compression_config": spec,
            "performance_metrics": {"compression_ratio": float(e["compression_ratio"]),
                                    "harmonic_speed_mbps": float(S),
                                    "critical_bandwidth_mbps":
                                        (1 - 1 / float(e["compression_ratio"])) * float(S)},
            "quality_metrics": {"accuracy": float(e["accuracy"])}})
    buckets = []
    edges = sorted(acc_edges)
    bw = sorted(bw_edges_mbps, reverse=True)  # high -> low bandwidth == low -> high x
    for bi in range(len(edges) - 1):
        lo, hi = edges[bi], edges[bi + 1]
        members = [p for p in profiles if p["quality_metrics"]["accuracy"] >= lo]
        pareto = _pareto(members)
        intervals = []
        for ii in range(len(bw) - 1):
            b_hi, b_lo = bw[ii], bw[ii + 1]
            mid = math.sqrt(b_hi * b_lo)

            def lat(p):  # seconds per MB of KV
                pm = p["performance_metrics"]
                return 1 / pm["harmonic_speed_mbps"] + 1 / (pm["compression_ratio"] * mid)
            ranked = sorted((p for p in pareto if lat(p) < 1 / mid), key=lat)
            intervals.append({"interval_id": ii, "x_range": [1 / b_hi, 1 / b_lo],
                              "candidate_profile_ids": [p["profile_id"] for p in ranked[:k]],
                              "model_optimal_profile_id": ranked[0]["profile_id"] if ranked else None})
        # beyond the lowest bandwidth edge
        intervals.append({"interval_id": len(bw) - 1, "x_range": [1 / bw[-1], float("inf")],
                          "candidate_profile_ids": [p["profile_id"] for p in sorted(
                              pareto, key=lambda p: -p["performance_metrics"]["compression_ratio"])[:k]]})
        buckets.append({"bucket_id": bi, "acc_range": [lo, hi], "pareto_profiles": pareto,
                        "bandwidth_intervals": intervals})
    return {"library_metadata": {"model_name": model_name, "dataset": dataset,
                                 "generator": "kvserve_hpdps_b200.offline.library_export"},
            "accuracy_buckets": buckets}


def write_library(path: str, library: dict) -> None:
    def fix(o):
        if isinstance(o, float) and math.isinf(o):
            return 1e30
        if isinstance(o, dict):
            return {k: fix(v) for k, v in o.items()}
        if isinstance(o, list):
            return [fix(v) for v in o]
        return o
    with open(path, "w") as f:
        json.dump(fix(library), f, indent=2)
