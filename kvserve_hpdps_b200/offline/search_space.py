"""Search space of the offline profile search.

A candidate is a quantizer configuration (reference search space:
kvserve_v1/offline_search/evaluation/param_search/test_search.py:25-56):
``hybrid_ratio`` (fraction of (layer, head) pairs at LOW precision), the four
level counts (high/low x key/value), the key/value axes and the split type.
Valid candidates have low <= high for keys and values.
"""

from __future__ import annotations

import itertools
from dataclasses import asdict, dataclass
from typing import Iterable, Optional

DEFAULT_SPACE = {
    "hybrid_ratio": [0.0, 0.3, 0.5, 0.8, 1.0],
    "high_key_max_value": [16, 12, 8],
    "high_value_max_value": [16, 12, 8],
    "low_key_max_value": [12, 8, 6, 4],
    "low_value_max_value": [8, 6, 4],
    "axis_key": ["channel"],
    "axis_value": ["token"],
    "split_type": ["head"],
}


@dataclass(frozen=True)
class Candidate:
    hybrid_ratio: float
    high_key_max_value: int
    high_value_max_value: int
    low_key_max_value: int
    low_value_max_value: int
    axis_key: str = "channel"
    axis_value: str = "token"
    split_type: str = "head"

    def quantizer_config(self, model_name: Optional[str] = None) -> dict:
        d = asdict(self)
        if model_name:
            d["model_name"] = model_name
        return d

    def key(self) -> str:
        return (f"hr{self.hybrid_ratio}_k{self.high_key_max_value}-{self.low_key_max_value}"
                f"_v{self.high_value_max_value}-{self.low_value_max_value}"
                f"_{self.axis_key[0]}{self.axis_value[0]}_{self.split_type}")

    def vector(self) -> list[float]:
        """Numeric features for the surrogate model (levels as bits)."""
        import math
        return [self.hybrid_ratio, math.log2(self.high_key_max_value),
                math.log2(self.high_value_max_value), math.log2(self.low_key_max_value),
                math.log2(self.low_value_max_value)]

    def dominates_in_precision(self, other: "Candidate") -> bool:
        """True when self keeps at least as much precision as ``other`` in
        every dimension (fewer low heads and more levels everywhere)."""
        return (self.hybrid_ratio <= other.hybrid_ratio
                and self.high_key_max_value >= other.high_key_max_value
                and self.high_value_max_value >= other.high_value_max_value
                and self.low_key_max_value >= other.low_key_max_value
                and self.low_value_max_value >= other.low_value_max_value
                and (self.axis_key, self.axis_value, self.split_type) ==
                (other.axis_key, other.axis_value, other.split_type))


def is_valid(c: Candidate) -> bool:
    return (c.low_key_max_value <= c.high_key_max_value
            and c.low_value_max_value <= c.high_value_max_value
            and 0.0 <= c.hybrid_ratio <= 1.0
            and all(1 < v < 255 for v in (c.high_key_max_value, c.high_value_max_value,
                                          c.low_key_max_value, c.low_value_max_value)))


def enumerate_space(space: Optional[dict] = None) -> list[Candidate]:
    sp = dict(DEFAULT_SPACE)
    sp.update(space or {})
    keys = list(sp)
    out = []
    for vals in itertools.product(*(sp[k] for k in keys)):
        c = Candidate(**dict(zip(keys, vals)))
        if is_valid(c):
            out.append(c)
    return out


def prune_after(result_candidate: Candidate, feasible: bool,
                pool: Iterable[Candidate]) -> list[Candidate]:
    """Dominance pruning: if a candidate misses the accuracy target, every
    candidate with no more precision anywhere misses it too; if it meets the
    target, every candidate with at least as much precision everywhere has no
    better compression ratio.  Returns the pool minus the pruned ones."""
    keep = []
    for c in pool:
        if c == result_candidate:
            continue
        if not feasible and result_candidate.dominates_in_precision(c):
            continue
        if feasible and c.dominates_in_precision(result_candidate):
            continue
        keep.append(c)
    return keep
