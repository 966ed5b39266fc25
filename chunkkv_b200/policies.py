"""Cache policies P0-P4 as runtimes over one engine (drop-in for the reference's
bench/policies.py:1-35, with this package's store, gate and runtimes).

P0  no cache (full recompute)               ChunkReuseRuntime(enabled=False)
P1  exact prefix cache                      PrefixCacheRuntime
P2  naive chunk reuse, token-keyed          gate mode "naive", provenance off
P3  CacheBlend-style fixed recompute        gate mode "always_blend" at `ratio`, provenance off
P4  ChunkKV: gate + provenance keys         gate "gated", ratios (ratio, min(1, 2 ratio))
"""

from __future__ import annotations

from chunkkv_b200.gate import GateConfig, ReuseGate
from chunkkv_b200.runtime import ChunkReuseRuntime, PrefixCacheRuntime
from chunkkv_b200.store.kvstore import KVStore

POLICIES = ["P0", "P1", "P2", "P3", "P4"]
DESCRIPTIONS = {
    "P0": "no cache (full recompute)",
    "P1": "exact prefix cache",
    "P2": "naive chunk reuse, token-keyed",
    "P3": "CacheBlend-style fixed recompute, token-keyed",
    "P4": "ChunkKV: gate + provenance keys",
}


# policy -> (runtime kind, gate settings as GateConfig fields, runtime options).
# Ratios are written in units of the `ratio` argument: ("ratio", k) means
# min(1, k * ratio).  The settings are bench/policies.py:20-35's.
_TABLE: dict[str, tuple[str, dict, dict]] = {
    "P0": ("chunk", {}, {"enabled": False}),
    "P1": ("prefix", {}, {}),
    "P2": ("chunk", {"mode": "naive"}, {"provenance": False}),
    "P3": ("chunk", {"mode": "always_blend", "ratio_same_context": ("ratio", 1)}, {"provenance": False}),
    "P4": ("chunk", {"ratio_same_context": ("ratio", 1), "ratio_other_context": ("ratio", 2),
                     "escalate_threshold": "escalate", "cross_context": "cross_context"}, {"provenance": True}),
}


def build(policy: str, engine, model_id: str, budget_bytes: int = 3 << 30, ratio: float = 0.15,
          escalate: float | None = None, cross_context: str = "blend", store: KVStore | None = None):
    """The runtime for `policy`.  `store` (optional) replaces the fresh KVStore of
    `budget_bytes` that the chunk-reuse policies get by default."""
    if policy not in _TABLE:
        raise ValueError(policy)
    kind, gate_fields, opts = _TABLE[policy]
    if kind == "prefix":
        return PrefixCacheRuntime(engine, budget_bytes)
    args = {"escalate": escalate, "cross_context": cross_context}

    def value(v):
        if isinstance(v, tuple):  # ("ratio", k)
            return ratio if v[1] == 1 else min(1.0, v[1] * ratio)
        return args[v] if isinstance(v, str) and v in args else v

    gate = ReuseGate(GateConfig(**{k: value(v) for k, v in gate_fields.items()}))
    store = store if store is not None else KVStore(budget_bytes, device=getattr(engine, "device", None))
    return ChunkReuseRuntime(engine, model_id, store, gate, **opts)
