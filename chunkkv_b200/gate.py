"""Reuse gate (drop-in for chunkkv.gate.gate, src/chunkkv/gate/gate.py:1-76).

For each reusable segment that has stored variants, the gate picks one variant
and an action: REUSE (serve unchanged), BLEND (serve with selective recompute at
a ratio) or RECOMPUTE (serve nothing).  Here the policy is data: each mode is an
ordered table of rules, and a rule is "the first candidate variant that satisfies
this predicate, served with this action at the ratio held in this config field".
Candidates are all variants, except in the "gated" mode, which first drops the
variants computed after less-trusted content than the request holds before the
segment (reason "trust" when none is left).

The tables restate the reference's decision order, reasons and ratios
(gate.py:38-72), which the runtime parity tests compare call by call:

  gated        exact_prefix -> REUSE;  same_context -> BLEND ratio_same_context;
               other_context -> BLEND ratio_other_context, or RECOMPUTE when
               cross_context == "recompute"
  always_blend exact_prefix -> REUSE;  fixed -> BLEND ratio_same_context  (P3)
  naive        exact_prefix -> REUSE;  naive -> BLEND at ratio 0          (P2)

`decide` has the reference's signature and hashes the request prefix itself;
`decide_hashed` takes the prefix hash and the trust floor from a runtime that
computed them once per request (chunkkv_b200.runtime.RequestHashes).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Literal, NamedTuple

from chunkkv_b200.store.keys import token_hash
from chunkkv_b200.types import ChunkedRequest, GateAction, GateDecision, Segment, TrustLevel


@dataclass
class GateConfig:
    """Same fields and defaults as the reference's GateConfig (gate.py:26-32)."""

    mode: Literal["gated", "always_blend", "naive"] = "gated"
    ratio_same_context: float = 0.10
    ratio_other_context: float = 0.20
    cross_context: Literal["blend", "recompute"] = "blend"
    escalate_threshold: float | None = 0.5  # relative layer-1 deviation (BlendConfig)


class _Probe(NamedTuple):
    """What a rule can compare a stored variant with."""

    prefix_hash: str
    context_id: str


@dataclass(frozen=True)
class Rule:
    reason: str
    serves: Callable[[object, _Probe], bool]   # (entry, probe) -> may this rule serve it
    action: GateAction
    ratio_field: str | None = None              # GateConfig field with the ratio (None: 0.0)
    recompute_if: tuple[str, str] | None = None  # (GateConfig field, value) that turns it into RECOMPUTE


def _same_prefix(e, p: _Probe) -> bool:
    return e.prefix_hash == p.prefix_hash


def _same_context(e, p: _Probe) -> bool:
    return e.context_id == p.context_id


def _any(e, p: _Probe) -> bool:
    return True


_EXACT = Rule("exact_prefix", _same_prefix, GateAction.REUSE)
RULES: dict[str, tuple[Rule, ...]] = {
    "gated": (
        _EXACT,
        Rule("same_context", _same_context, GateAction.BLEND, "ratio_same_context"),
        Rule("other_context", _any, GateAction.BLEND, "ratio_other_context",
             recompute_if=("cross_context", "recompute")),
    ),
    "always_blend": (_EXACT, Rule("fixed", _any, GateAction.BLEND, "ratio_same_context")),
    "naive": (_EXACT, Rule("naive", _any, GateAction.BLEND)),
}
# modes whose candidates must pass the trust floor first
TRUST_FILTERED = frozenset({"gated"})


class ReuseGate:
    def __init__(self, config: GateConfig | None = None):
        self.config = config or GateConfig()
        self.log: list[GateDecision] = []

    def decide(self, req: ChunkedRequest, seg: Segment, entries: list) -> tuple[GateDecision, object | None]:
        return self.decide_hashed(req, seg, entries, token_hash(req.tokens[: seg.start]),
                                  req.context_trust_before(seg.start))

    def decide_hashed(self, req: ChunkedRequest, seg: Segment, entries: list, prefix_hash: str,
                      trust_floor: TrustLevel) -> tuple[GateDecision, object | None]:
        cfg = self.config
        rules = RULES.get(cfg.mode)
        if rules is None:
            raise ValueError(f"unknown gate mode {cfg.mode!r}")
        candidates = entries
        if cfg.mode in TRUST_FILTERED:
            candidates = [e for e in entries if e.context_trust >= trust_floor]
            if not candidates:
                return self._record(GateDecision(seg.index, GateAction.RECOMPUTE, "trust"), None)
        probe = _Probe(prefix_hash, req.context_id)
        for rule in rules:
            hit = next((e for e in candidates if rule.serves(e, probe)), None)
            if hit is None:
                continue
            if rule.recompute_if is not None and getattr(cfg, rule.recompute_if[0]) == rule.recompute_if[1]:
                return self._record(GateDecision(seg.index, GateAction.RECOMPUTE, rule.reason), None)
            ratio = getattr(cfg, rule.ratio_field) if rule.ratio_field else 0.0
            return self._record(GateDecision(seg.index, rule.action, rule.reason, ratio, hit.id), hit)
        # every table ends in a rule that serves any candidate, so this is only
        # reached with no stored variants at all (the runtime never asks then)
        return self._record(GateDecision(seg.index, GateAction.RECOMPUTE, "no_entries"), None)

    def _record(self, d: GateDecision, entry):
        self.log.append(d)
        return d, entry
