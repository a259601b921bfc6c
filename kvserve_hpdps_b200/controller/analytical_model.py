"""Analytical latency model of a compressed transfer.

T_p = T_model + V/S + V/(cr*B) with compression, T_0 = T_model + V/B without
(V in MB, S and B in MB/s, cr = original/compressed).  Compression is
beneficial iff B < (1 - 1/cr) * S (Theorem 1).

The reference's predictor multiplies V by cr in the transfer term
(kvserve_v1/compression/controller/analytical_model.py:58-59), which
contradicts both its own docstring and the benefit test; this model uses
V/(cr*B).  ``reference_transfer_term=True`` reproduces the reference's
expression for comparisons.
"""

from __future__ import annotations

from kvserve_hpdps_b200.controller.profile import Profile

MB = 1024 * 1024


class AnalyticalModel:
    def __init__(self, reference_transfer_term: bool = False):
        self.reference_transfer_term = reference_transfer_term

    def predict_latency(self, profile: Profile, V_bytes: float, B_mbps: float,
                        T_model_ms: float) -> float:
        V = V_bytes / MB
        cr = profile.compression_ratio
        t_codec = V / profile.harmonic_speed * 1e3
        moved = V * cr if self.reference_transfer_term else V / cr
        return T_model_ms + t_codec + moved / B_mbps * 1e3

    @staticmethod
    def predict_baseline_latency(V_bytes: float, B_mbps: float, T_model_ms: float) -> float:
        return T_model_ms + (V_bytes / MB) / B_mbps * 1e3

    @staticmethod
    def check_benefit(profile: Profile, B_mbps: float) -> bool:
        cr, S = profile.compression_ratio, profile.harmonic_speed
        return B_mbps < (1 - 1 / cr) * S

    def compute_speedup(self, profile: Profile, V_bytes: float, B_mbps: float,
                        T_model_ms: float) -> float:
        return (self.predict_baseline_latency(V_bytes, B_mbps, T_model_ms)
                / self.predict_latency(profile, V_bytes, B_mbps, T_model_ms))
