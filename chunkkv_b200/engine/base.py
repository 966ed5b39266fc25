"""Request types of the blend prefill (drop-in for chunkkv.engine.base).

The names, fields and defaults are the reference's data contract
(src/chunkkv/engine/base.py:13-73): K/V are (1, n_kv_heads, L, head_dim) per
layer with RoPE applied, ChunkKV.start is the position the chunk was computed
at, Placement.start the position it is served at.  `plan_arrays` is the
vectorised planner the CUDA engine uses; `plan_positions` keeps the
reference's list-returning signature on top of it.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable

import numpy as np


@dataclass
class ChunkKV:
    """Per-layer K/V of one chunk, computed at positions start .. start+length."""

    keys: list[Any]
    values: list[Any]
    start: int

    @property
    def length(self) -> int:
        return self.keys[0].shape[2]


class CacheChunkKV:
    """ChunkKV of a CUDA-engine result: positions [start, end) of its blended cache
    (two [L, H, N, D] tensors).  `keys` / `values` are the reference's per-layer
    (1, H, len, D) tensors, copied out on first access so that a chunk kept by the
    caller stops pinning the request's cache (base.py:53 of the reference copies
    eagerly).  Until then the chunk is a view: this package's KVStore writes its
    pages, and the engine gathers, straight from the cache without the L x 2 copies."""

    def __init__(self, cache, start: int, end: int, copy: Callable[[Any], Any]):
        self._cache = cache
        self.start = start
        self._end = end
        self._copy = copy
        self._kv: tuple[list[Any], list[Any]] | None = None

    @property
    def length(self) -> int:
        return self._end - self.start

    @property
    def viewable(self) -> bool:
        return self._cache is not None

    @property
    def n_layers(self) -> int:
        return self._cache[0].shape[0] if self._cache is not None else len(self._kv[0])

    def view(self, li: int, kv: int):
        """(H, len, D) view of layer `li` (kv 0: K, 1: V) in the cache."""
        return self._cache[kv][li, :, self.start:self._end]

    def _materialise(self):
        if self._kv is None:
            K, V = self._cache
            L = K.shape[0]
            self._kv = ([self._copy(K[li, None, :, self.start:self._end]) for li in range(L)],
                        [self._copy(V[li, None, :, self.start:self._end]) for li in range(L)])
            self._cache = None
        return self._kv

    @property
    def keys(self) -> list[Any]:
        return self._materialise()[0]

    @property
    def values(self) -> list[Any]:
        return self._materialise()[1]


@dataclass
class Placement:
    """A cached chunk served at a new offset `start` of the request."""

    chunk: Any  # ChunkKV or store.pages.PagedChunkKV
    start: int
    ratio: float | None = None  # per-chunk recompute ratio; None = BlendConfig.recompute_ratio
    exact: bool = False         # computed after the same prefix: never recomputed, not even at layer 0


@dataclass
class BlendConfig:
    recompute_ratio: float = 0.15  # share of cached tokens recomputed at layers >= 1
    n_sink: int = 2                # first tokens of every moved chunk, always recomputed
    full_first_layer: bool = True  # False = naive reuse (no repair)
    # Deviation probe: a chunk whose relative layer-1 K/V deviation exceeds this
    # is recomputed whole from layer 1 on.  None disables the probe.
    escalate_threshold: float | None = None


@dataclass
class PrefillResult:
    logits: Any            # (n, vocab) for the positions in logit_positions
    logit_positions: Any
    keys: list[Any]        # full K per layer for the whole request, (1, H, N, D)
    values: list[Any]
    stats: dict = field(default_factory=dict)
    copy: Callable[[Any], Any] = lambda a: a  # so stored chunks do not pin request buffers
    # CUDA engine extras: the blended cache as two [L, H, N, D] tensors (keys/values
    # are views of them) and selection details.  None for results of other engines.
    cache: tuple[Any, Any] | None = None
    selected: Any = None   # ascending positions recomputed at layers >= 1 (int32)

    def chunk(self, start: int, end: int) -> ChunkKV:
        if self.cache is not None:
            return CacheChunkKV(self.cache, start, end, self.copy)
        return ChunkKV(
            keys=[self.copy(k[:, :, start:end, :]) for k in self.keys],
            values=[self.copy(v[:, :, start:end, :]) for v in self.values],
            start=start,
        )


@dataclass
class Plan:
    """Per-position flags of one request plus the index lists derived from them."""

    n: int
    cached: np.ndarray   # bool [n]
    exact: np.ndarray    # bool [n]
    sink: np.ndarray     # bool [n]

    @property
    def fresh_idx(self) -> np.ndarray:
        return np.flatnonzero(~self.cached).astype(np.int32)

    @property
    def layer0_idx(self) -> np.ndarray:
        return np.flatnonzero(~self.exact).astype(np.int32)

    def pos_flags(self) -> np.ndarray:
        """uint8 [n]: bit0 cached, bit1 sink, bit2 exact (the selection kernel's input)."""
        return (self.cached.astype(np.uint8) | (self.sink.astype(np.uint8) << 1)
                | (self.exact.astype(np.uint8) << 2))


def plan_arrays(n: int, placements: list[Placement], n_sink: int) -> Plan:
    """Vectorised plan_positions: later placements OR into earlier ones, as the reference's loop does."""
    cached = np.zeros(n, dtype=bool)
    exact = np.zeros(n, dtype=bool)
    sink = np.zeros(n, dtype=bool)
    for p in placements:
        s, e = p.start, p.start + p.chunk.length
        if s < 0 or e > n:
            raise IndexError(f"placement [{s}, {e}) lies outside the request of {n} tokens")
        cached[s:e] = True
        if p.exact:
            exact[s:e] = True
        else:
            sink[s:min(e, s + max(0, n_sink))] = True
    return Plan(n, cached, exact, sink)


def plan_positions(n: int, placements: list[Placement], n_sink: int):
    """Per-position flags as python lists: cached, exact, sink (base.py:63-73 contract)."""
    plan = plan_arrays(n, placements, n_sink)
    return plan.cached.tolist(), plan.exact.tolist(), plan.sink.tolist()
