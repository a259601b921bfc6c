"""A compression profile: a pipeline config with measured performance.

JSON form (profile-library schema, reference profile.py:38-44):
``{"profile_id", "metadata", "compression_config", "performance_metrics":
{"compression_ratio", "harmonic_speed_mbps", "critical_bandwidth_mbps"?},
"quality_metrics": {"accuracy"}}``.  ``compression_ratio`` is original /
compressed (> 1); the harmonic speed S = S_enc*S_dec/(S_enc+S_dec) is in MB/s
of original KV.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any


@dataclass
class Profile:
    profile_id: str
    compression_config: dict[str, Any]
    performance_metrics: dict[str, float]
    quality_metrics: dict[str, float]
    metadata: dict[str, Any] = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "Profile":
        return cls(profile_id=d["profile_id"], compression_config=d["compression_config"],
                   performance_metrics=d["performance_metrics"],
                   quality_metrics=d["quality_metrics"], metadata=d.get("metadata", {}))

    def to_dict(self) -> dict[str, Any]:
        return {"profile_id": self.profile_id, "metadata": self.metadata,
                "compression_config": self.compression_config,
                "performance_metrics": self.performance_metrics,
                "quality_metrics": self.quality_metrics}

    @property
    def compression_ratio(self) -> float:
        return float(self.performance_metrics["compression_ratio"])

    @property
    def harmonic_speed(self) -> float:
        return float(self.performance_metrics["harmonic_speed_mbps"])

    @property
    def critical_bandwidth(self) -> float:
        """B_crit = (1 - 1/cr) * S: compression pays off below this bandwidth."""
        return float(self.performance_metrics.get(
            "critical_bandwidth_mbps", (1 - 1 / self.compression_ratio) * self.harmonic_speed))

    @property
    def accuracy(self) -> float:
        return float(self.quality_metrics["accuracy"])

    def __repr__(self) -> str:
        return f"Profile(id={self.profile_id}, cr={self.compression_ratio:.2f}, acc={self.accuracy:.3f})"
