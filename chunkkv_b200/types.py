"""Request-level types used by the store and the runtime (drop-in for chunkkv.types).

Same names, fields and semantics as src/chunkkv/types.py:9-59 of the reference,
so store entries and gate decisions can be passed between the two.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum, IntEnum


class TrustLevel(IntEnum):
    """Who controls a piece of content; a larger value is more trusted."""

    USER = 0
    TOOL = 1
    SYSTEM = 2


class GateAction(str, Enum):
    REUSE = "reuse"          # serve cached K/V unchanged (same preceding tokens)
    BLEND = "blend"          # serve with selective recompute
    RECOMPUTE = "recompute"  # do not serve; prefill from scratch


@dataclass
class Segment:
    """A contiguous, possibly reusable span of request tokens."""

    index: int
    role: str
    trust: TrustLevel
    start: int
    tokens: list[int]
    reusable: bool = True

    @property
    def end(self) -> int:
        return self.start + len(self.tokens)


@dataclass
class ChunkedRequest:
    tokens: list[int]
    segments: list[Segment]
    tenant_id: str
    context_id: str

    def context_trust_before(self, pos: int) -> TrustLevel:
        """Lowest trust among the segments that start before `pos` (SYSTEM if none)."""
        before = [s.trust for s in self.segments if s.start < pos]
        return min(before) if before else TrustLevel.SYSTEM


@dataclass
class GateDecision:
    segment: int
    action: GateAction
    reason: str
    ratio: float = 0.0
    entry_id: str | None = None
    extra: dict = field(default_factory=dict)
