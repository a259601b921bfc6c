"""Profile library: accuracy buckets x bandwidth intervals (in 1/B space)
of Pareto-candidate profiles.

Schema (reference profile_library.py:44-77)::

  {"library_metadata": {...},
   "accuracy_buckets": [{"bucket_id", "acc_range": [lo, hi],
       "pareto_profiles": [<profile>...],
       "bandwidth_intervals": [{"interval_id", "x_range": [1/B_hi, 1/B_lo],
           "candidate_profile_ids": [...], "model_optimal_profile_id"?}]}]}

Lookups fall back to the closest bucket and to the last (lowest-bandwidth)
interval, as the reference does.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Optional

from kvserve_hpdps_b200.controller.profile import Profile


class ProfileLibrary:
    def __init__(self, json_path: Optional[str] = None, data: Optional[dict] = None):
        if data is None:
            if json_path is None or not Path(json_path).exists():
                raise FileNotFoundError(f"profile library not found: {json_path}")
            with open(json_path) as f:
                data = json.load(f)
        self.metadata = data.get("library_metadata", {})
        self.accuracy_buckets: list[dict] = data.get("accuracy_buckets", [])
        self.profile_map: dict[str, Profile] = {}
        for b in self.accuracy_buckets:
            for pd in b.get("pareto_profiles", []):
                p = Profile.from_dict(pd)
                self.profile_map[p.profile_id] = p
        self._validate()

    def _validate(self) -> None:
        if not self.accuracy_buckets:
            raise ValueError("profile library has no accuracy buckets")
        for b in self.accuracy_buckets:
            for key in ("bucket_id", "acc_range", "bandwidth_intervals"):
                if key not in b:
                    raise ValueError(f"bucket missing {key!r}")

    def find_bucket(self, acc_req: float) -> Optional[dict]:
        for b in self.accuracy_buckets:
            lo, hi = b["acc_range"]
            if lo <= acc_req < hi:
                return b
        if not self.accuracy_buckets:
            return None
        return min(self.accuracy_buckets,
                   key=lambda b: min(abs(b["acc_range"][0] - acc_req),
                                     abs(b["acc_range"][1] - acc_req)))

    def find_interval(self, bucket: dict, B_mbps: float) -> Optional[dict]:
        x = 1.0 / B_mbps
        ints = bucket.get("bandwidth_intervals", [])
        for it in ints:
            lo, hi = it["x_range"]
            if lo <= x < hi:
                return it
        return ints[-1] if ints else None

    def get_profile(self, profile_id: str) -> Optional[Profile]:
        return self.profile_map.get(profile_id)

    def get_candidate_profiles(self, bucket: dict, interval: dict) -> list[Profile]:
        return [self.profile_map[p] for p in interval.get("candidate_profile_ids", [])
                if p in self.profile_map]

    def get_optimal_profile(self, bucket: dict, interval: dict) -> Optional[Profile]:
        pid = interval.get("model_optimal_profile_id")
        return self.get_profile(pid) if pid else None

    def get_all_profiles(self) -> list[Profile]:
        return list(self.profile_map.values())

    def get_num_profiles(self) -> int:
        return len(self.profile_map)

    def get_num_buckets(self) -> int:
        return len(self.accuracy_buckets)

    def get_bucket_info(self, bucket_id: int) -> Optional[dict]:
        return next((b for b in self.accuracy_buckets if b["bucket_id"] == bucket_id), None)

    def summary(self) -> str:
        n_int = sum(len(b.get("bandwidth_intervals", [])) for b in self.accuracy_buckets)
        return (f"ProfileLibrary(model={self.metadata.get('model_name', '?')}, "
                f"profiles={self.get_num_profiles()}, buckets={self.get_num_buckets()}, "
                f"intervals={n_int})")
