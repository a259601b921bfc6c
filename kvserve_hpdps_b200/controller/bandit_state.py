"""Per-(bucket, interval, profile) residual statistics of the bandit.

State: key -> (N, delta_bar) with delta_bar an EWMA of residuals
T_obs - T_hat: delta_bar <- (1 - alpha) * delta_bar + alpha * delta.
JSON persistence uses keys ``"<bucket>_<interval>_<profile_id>"`` (reference
bandit_state.py:109-157), so state files move between the two.
"""

from __future__ import annotations

import json
import os
from pathlib import Path


class BanditStateManager:
    def __init__(self, alpha: float = 0.2):
        if not 0 < alpha <= 1:
            raise ValueError("alpha must be in (0, 1]")
        self.alpha = alpha
        self.state: dict[tuple[int, int, str], tuple[int, float]] = {}

    def get_stats(self, bucket_id: int, interval_id: int, profile_id: str) -> tuple[int, float]:
        return self.state.get((bucket_id, interval_id, profile_id), (0, 0.0))

    def update(self, bucket_id: int, interval_id: int, profile_id: str, delta_obs: float) -> None:
        key = (bucket_id, interval_id, profile_id)
        n, d = self.state.get(key, (0, 0.0))
        self.state[key] = (n + 1, (1 - self.alpha) * d + self.alpha * delta_obs)

    def get_usage_count(self, b: int, i: int, p: str) -> int:
        return self.get_stats(b, i, p)[0]

    def get_residual(self, b: int, i: int, p: str) -> float:
        return self.get_stats(b, i, p)[1]

    def reset(self) -> None:
        self.state.clear()

    def save(self, path: str) -> None:
        data = {"alpha": self.alpha,
                "state": {f"{b}_{i}_{p}": {"N": n, "delta_bar": d}
                          for (b, i, p), (n, d) in self.state.items()}}
        Path(path).parent.mkdir(parents=True, exist_ok=True)
        tmp = f"{path}.tmp"
        with open(tmp, "w") as f:
            json.dump(data, f, indent=2)
        os.replace(tmp, path)

    def load(self, path: str) -> None:
        with open(path) as f:
            data = json.load(f)
        self.alpha = float(data["alpha"])
        self.state = {}
        for key, st in data["state"].items():
            parts = key.split("_", 2)
            if len(parts) == 3:
                self.state[(int(parts[0]), int(parts[1]), parts[2])] = (int(st["N"]),
                                                                        float(st["delta_bar"]))

    def get_total_states(self) -> int:
        return len(self.state)

    def get_memory_size(self) -> int:
        return 60 * len(self.state)
