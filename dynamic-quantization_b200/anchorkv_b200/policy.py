"""Cache representation modes and the plan type the block store applies.

Mirrors the parts of ``src/anchorkv/policy.py`` the block store depends on:
``CacheMode`` (policy.py:12-18) and the ``PlannedSegment`` / ``CachePlan``
records ``DeclarativeKVCache.apply_plan`` consumes (policy.py:140-161).  The
planner itself (anchor tracking, byte-budget search) is host-side research
tooling outside the packed decode path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from enum import Enum


class CacheMode(str, Enum):
    """Storage representation of a block, in decreasing precision order."""

    EVICTED = "evicted"
    INT4 = "int4"
    INT8 = "int8"
    FP16 = "fp16"


# Lifecycle rank: a block may only move to a lower rank (backend.py:455-460).
PRECISION_RANK = {CacheMode.EVICTED: 0, CacheMode.INT4: 1, CacheMode.INT8: 2, CacheMode.FP16: 3}


def as_mode(mode) -> CacheMode:
    """Accept this module's CacheMode, the reference's (same values) or a string."""
    if isinstance(mode, CacheMode):
        return mode
    return CacheMode(getattr(mode, "value", mode))


@dataclass(frozen=True, slots=True)
class PlannedSegment:
    segment_id: int
    mode: CacheMode
    bytes_used: int
    importance: float
    reason: str


@dataclass(frozen=True, slots=True)
class CachePlan:
    segments: tuple[PlannedSegment, ...]
    budget_bytes: int
    used_bytes: int
    full_cache_bytes: int

    @property
    def compression_ratio(self) -> float:
        if self.used_bytes == 0:
            return math.inf if self.full_cache_bytes else 1.0
        return self.full_cache_bytes / self.used_bytes

    @property
    def budget_utilization(self) -> float:
        """Planned bytes over the budget (0 without a budget), policy.py:163-165."""
        return self.used_bytes / self.budget_bytes if self.budget_bytes else 0.0
