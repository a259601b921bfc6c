"""Constraint-aware Bayesian optimisation over the candidate space.

Goal: the highest compression ratio whose accuracy stays within
``tolerance`` (percentage points, relative to the uncompressed baseline) --
the reference's search (kvserve_v1/offline_search/evaluation/param_search/
test_search.py:237-601).  Procedure:

1. cold start: evaluate the candidates with the highest, median and lowest
   predicted compression (predicted from bits per element);
2. loop: fit a Gaussian process (Matern nu=1.5 + white noise) to accuracy
   over the evaluated candidates; score the remaining ones with
   ``cr_pred * P(accuracy >= threshold) + kappa * sigma``; evaluate the best;
3. after each evaluation prune dominated candidates (``prune_after``) and
   stop after ``patience`` evaluations without a better feasible CR or when
   the budget is spent.

The evaluation function is injected, so the driver runs on any evaluator
(the KV evaluator here, a model-based one elsewhere).
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from typing import Callable, Optional, Sequence

import numpy as np

from kvserve_hpdps_b200.offline.search_space import Candidate, prune_after


def predicted_bits(c: Candidate) -> float:
    """Bits per element before entropy coding (mean over K and V)."""
    hr = c.hybrid_ratio
    kb = hr * math.log2(c.low_key_max_value) + (1 - hr) * math.log2(c.high_key_max_value)
    vb = hr * math.log2(c.low_value_max_value) + (1 - hr) * math.log2(c.high_value_max_value)
    return (kb + vb) / 2


def predicted_cr(c: Candidate) -> float:
    return 16.0 / predicted_bits(c)


@dataclass
class SearchRecord:
    candidate: Candidate
    accuracy: float
    compression_ratio: float
    feasible: bool
    extra: dict = field(default_factory=dict)


class ConstraintAwareBO:
    def __init__(self, candidates: Sequence[Candidate], evaluate: Callable[[Candidate], dict],
                 threshold: float, budget: int = 20, patience: int = 6, kappa: float = 0.1,
                 seed: int = 0):
        self.pool = list(candidates)
        self.evaluate_fn = evaluate
        self.threshold = float(threshold)
        self.budget = int(budget)
        self.patience = int(patience)
        self.kappa = float(kappa)
        self.rng = np.random.default_rng(seed)
        self.history: list[SearchRecord] = []

    def _eval(self, c: Candidate) -> SearchRecord:
        res = self.evaluate_fn(c)
        acc = float(res["accuracy"])
        rec = SearchRecord(c, acc, float(res["compression_ratio"]), acc >= self.threshold,
                           {k: v for k, v in res.items() if k not in ("accuracy", "compression_ratio")})
        self.history.append(rec)
        self.pool = prune_after(c, rec.feasible, self.pool)
        return rec

    def _cold_start(self) -> list[Candidate]:
        order = sorted(self.pool, key=predicted_cr)
        picks = [order[-1], order[len(order) // 2], order[0]] if order else []
        out = []
        for p in picks:
            if p not in out:
                out.append(p)
        return out

    def _propose(self) -> Optional[Candidate]:
        if not self.pool:
            return None
        from sklearn.gaussian_process import GaussianProcessRegressor
        from sklearn.gaussian_process.kernels import ConstantKernel, Matern, WhiteKernel
        X = np.array([r.candidate.vector() for r in self.history])
        y = np.array([r.accuracy for r in self.history])
        if len(self.history) < 2 or np.ptp(y) == 0:
            return max(self.pool, key=predicted_cr)
        kern = ConstantKernel(1.0) * Matern(length_scale=np.ones(X.shape[1]), nu=1.5) + \
            WhiteKernel(1e-4)
        gp = GaussianProcessRegressor(kernel=kern, normalize_y=True, random_state=0)
        gp.fit(X, y)
        P = np.array([c.vector() for c in self.pool])
        mu, sd = gp.predict(P, return_std=True)
        sd = np.maximum(sd, 1e-9)
        from scipy.stats import norm
        p_feas = norm.cdf((mu - self.threshold) / sd)
        cr = np.array([predicted_cr(c) for c in self.pool])
        score = cr * p_feas + self.kappa * sd * cr.max()
        return self.pool[int(np.argmax(score))]

    def run(self) -> dict:
        best: Optional[SearchRecord] = None
        stale = 0
        for c in self._cold_start():
            if len(self.history) >= self.budget:
                break
            if c in self.pool:
                r = self._eval(c)
                if r.feasible and (best is None or r.compression_ratio > best.compression_ratio):
                    best = r
        while len(self.history) < self.budget and stale < self.patience:
            c = self._propose()
            if c is None:
                break
            r = self._eval(c)
            if r.feasible and (best is None or r.compression_ratio > best.compression_ratio):
                best, stale = r, 0
            else:
                stale += 1
        return {
            "threshold": self.threshold,
            "evaluations": len(self.history),
            "best": None if best is None else self._rec_dict(best),
            "history": [self._rec_dict(r) for r in self.history],
        }

    @staticmethod
    def _rec_dict(r: SearchRecord) -> dict:
        return {"candidate": r.candidate.key(), "config": r.candidate.quantizer_config(),
                "accuracy": r.accuracy, "compression_ratio": r.compression_ratio,
                "feasible": r.feasible, **r.extra}


def save_results(path: str, results: dict) -> None:
    with open(path, "w") as f:
        json.dump(results, f, indent=2)
