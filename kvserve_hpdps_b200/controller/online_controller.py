"""Two-tier online controller (reference online_controller.py:18-288).

Tier 1 (analytical): accuracy bucket -> bandwidth interval (1/B space) ->
candidate profiles -> benefit filter B < (1 - 1/cr) S.
Tier 2 (bandit): T_eff = T_hat + delta_bar must meet the SLO; then
epsilon-greedy: explore a random feasible profile with probability epsilon,
otherwise exploit the minimum T_eff.  ``update(context, T_obs)`` feeds the
residual T_obs - T_hat back into the EWMA.  ``None`` (no compression) is
returned with a ``reason`` in the context.

The random generator can be seeded for reproducible decisions.
"""

from __future__ import annotations

import os
import random
from typing import Any, Optional

from kvserve_hpdps_b200.controller.analytical_model import AnalyticalModel
from kvserve_hpdps_b200.controller.bandit_state import BanditStateManager
from kvserve_hpdps_b200.controller.profile import Profile
from kvserve_hpdps_b200.controller.profile_library import ProfileLibrary


class OnlineController:
    def __init__(self, profile_library: ProfileLibrary, epsilon: float = 0.1,
                 bandit_state: Optional[BanditStateManager] = None, alpha: float = 0.2,
                 seed: Optional[int] = None, model: Optional[AnalyticalModel] = None):
        self.library = profile_library
        self.epsilon = float(epsilon)
        self.bandit = bandit_state or BanditStateManager(alpha=alpha)
        self.model = model or AnalyticalModel()
        self.rng = random.Random(seed)
        self.total_decisions = 0
        self.exploit_count = 0
        self.explore_count = 0
        self.no_compression_count = 0

    def select_profile(self, V_bytes: float, B_mbps: float, T_model_ms: float, T_SLO_ms: float,
                       acc_req: float) -> tuple[Optional[Profile], dict[str, Any]]:
        self.total_decisions += 1
        bucket = self.library.find_bucket(acc_req)
        if bucket is None:
            self.no_compression_count += 1
            return None, {"reason": "no_matching_bucket", "acc_req": acc_req}
        interval = self.library.find_interval(bucket, B_mbps)
        if interval is None:
            self.no_compression_count += 1
            return None, {"reason": "no_matching_interval", "B_mbps": B_mbps}
        candidates = self.library.get_candidate_profiles(bucket, interval)
        ids = {"bucket_id": bucket["bucket_id"], "interval_id": interval["interval_id"]}
        if not candidates:
            self.no_compression_count += 1
            return None, {"reason": "no_candidates", **ids}
        candidates = [p for p in candidates if self.model.check_benefit(p, B_mbps)]
        if not candidates:
            self.no_compression_count += 1
            return None, {"reason": "no_benefit", "B_mbps": B_mbps, **ids}
        base = self.model.predict_baseline_latency(V_bytes, B_mbps, T_model_ms)
        preds: dict[str, dict] = {}
        for p in candidates:
            t_hat = self.model.predict_latency(p, V_bytes, B_mbps, T_model_ms)
            _, d = self.bandit.get_stats(bucket["bucket_id"], interval["interval_id"], p.profile_id)
            t_eff = t_hat + d
            if t_eff <= T_SLO_ms:
                preds[p.profile_id] = {"profile": p, "T_hat": t_hat, "T_eff": t_eff,
                                       "delta_bar": d, "speedup": base / t_eff if t_eff else 0.0}
        if not preds:
            self.no_compression_count += 1
            return None, {"reason": "slo_violation", "T_SLO_ms": T_SLO_ms,
                          "candidates": [p.profile_id for p in candidates], **ids}
        if self.rng.random() < self.epsilon:
            action, sel = "explore", self.rng.choice(sorted(preds))
            self.explore_count += 1
        else:
            action, sel = "exploit", min(preds, key=lambda k: (preds[k]["T_eff"], k))
            self.exploit_count += 1
        pr = preds[sel]
        ctx = {**ids, "profile_id": sel, "T_hat": pr["T_hat"], "T_eff": pr["T_eff"],
               "delta_bar": pr["delta_bar"], "speedup_predicted": pr["speedup"], "action": action,
               "num_candidates": len(candidates), "baseline_latency": base, "V_bytes": V_bytes,
               "B_mbps": B_mbps, "T_model_ms": T_model_ms, "T_SLO_ms": T_SLO_ms}
        return pr["profile"], ctx

    def update(self, context: dict[str, Any], T_obs_ms: float) -> None:
        if "profile_id" not in context:
            return
        self.bandit.update(context["bucket_id"], context["interval_id"], context["profile_id"],
                           T_obs_ms - context["T_hat"])

    def get_statistics(self) -> dict[str, Any]:
        n = self.total_decisions
        ee = self.exploit_count + self.explore_count
        return {"total_decisions": n, "exploit_count": self.exploit_count,
                "explore_count": self.explore_count,
                "no_compression_count": self.no_compression_count,
                "compression_rate": (n - self.no_compression_count) / n if n else 0,
                "exploitation_rate": self.exploit_count / ee if ee else 0,
                "bandit_states": self.bandit.get_total_states(),
                "bandit_memory_bytes": self.bandit.get_memory_size()}

    def reset_statistics(self) -> None:
        self.total_decisions = self.exploit_count = self.explore_count = 0
        self.no_compression_count = 0

    def save_state(self, path: str) -> None:
        self.bandit.save(path)

    def load_state(self, path: str) -> None:
        self.bandit.load(path)

    def try_load_state(self, path: str) -> bool:
        """Load the bandit state if the file exists (resume after restart)."""
        if path and os.path.exists(path):
            self.bandit.load(path)
            return True
        return False
