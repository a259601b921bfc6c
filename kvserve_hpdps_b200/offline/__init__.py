"""Offline profile search: candidate space, evaluators, constraint-aware
Bayesian optimisation and export to the controller's profile library."""

from kvserve_hpdps_b200.offline.search_space import Candidate, enumerate_space, prune_after  # noqa: F401
