"""Reuse gate (drop-in for chunkkv.gate.gate, src/chunkkv/gate/gate.py:1-76).

Per reusable segment that has stored variants, decide REUSE / BLEND / RECOMPUTE.
The rules, their order, the reasons and the ratios are the reference's
(gate.py:38-72):

  mode "always_blend" / "naive" (policies P3 / P2): serve the variant computed
  after the same preceding tokens if there is one (REUSE, "exact_prefix"), else
  the first variant, blended at `ratio_same_context` ("fixed") or not repaired at
  all ("naive", ratio 0).

  mode "gated" (P4), in order:
    1. trust: only variants whose context trust is at least the lowest trust the
       request has before the segment; none left -> RECOMPUTE "trust";
    2. same preceding tokens -> REUSE "exact_prefix";
    3. same context id -> BLEND "same_context" at `ratio_same_context`;
    4. otherwise RECOMPUTE "other_context" when `cross_context="recompute"`, else
       BLEND "other_context" at `ratio_other_context` with the first allowed variant.

`decide` has the reference's signature and hashes the request prefix itself.
`decide_hashed` takes the prefix hash and the trust floor from the caller, so a
runtime that computed them once per request (chunkkv_b200.runtime) does no
per-segment O(request length) work here.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

from chunkkv_b200.store.keys import token_hash
from chunkkv_b200.types import ChunkedRequest, GateAction, GateDecision, Segment, TrustLevel


@dataclass
class GateConfig:
    mode: Literal["gated", "always_blend", "naive"] = "gated"
    ratio_same_context: float = 0.10
    ratio_other_context: float = 0.20
    cross_context: Literal["blend", "recompute"] = "blend"
    escalate_threshold: float | None = 0.5  # relative layer-1 deviation (BlendConfig)


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
        if cfg.mode != "gated":
            entry = next((e for e in entries if e.prefix_hash == prefix_hash), entries[0])
            if entry.prefix_hash == prefix_hash:
                d = GateDecision(seg.index, GateAction.REUSE, "exact_prefix", 0.0, entry.id)
            elif cfg.mode == "naive":
                d = GateDecision(seg.index, GateAction.BLEND, "naive", 0.0, entry.id)
            else:
                d = GateDecision(seg.index, GateAction.BLEND, "fixed", cfg.ratio_same_context, entry.id)
            return self._log(d), entry

        allowed = [e for e in entries if e.context_trust >= trust_floor]
        if not allowed:
            return self._log(GateDecision(seg.index, GateAction.RECOMPUTE, "trust")), None
        exact = next((e for e in allowed if e.prefix_hash == prefix_hash), None)
        if exact is not None:
            return self._log(GateDecision(seg.index, GateAction.REUSE, "exact_prefix", 0.0, exact.id)), exact
        same = next((e for e in allowed if e.context_id == req.context_id), None)
        if same is not None:
            d = GateDecision(seg.index, GateAction.BLEND, "same_context", cfg.ratio_same_context, same.id)
            return self._log(d), same
        if cfg.cross_context == "recompute":
            return self._log(GateDecision(seg.index, GateAction.RECOMPUTE, "other_context")), None
        entry = allowed[0]
        d = GateDecision(seg.index, GateAction.BLEND, "other_context", cfg.ratio_other_context, entry.id)
        return self._log(d), entry

    def _log(self, d: GateDecision) -> GateDecision:
        self.log.append(d)
        return d
