from __future__ import annotations

from kernelo_b200.tuning.cache import ConfigCache
from kernelo_b200.tuning.config import KernelConfig, Problem
from kernelo_b200.tuning.search import SearchSpace, search_space
from kernelo_b200.tuning.tuner import CandidateOutcome, Tuner, TuningResult

__all__ = [
    "CandidateOutcome",
    "ConfigCache",
    "KernelConfig",
    "Problem",
    "SearchSpace",
    "Tuner",
    "TuningResult",
    "search_space",
]
