"""Request path over the B200 engine and paged store (drop-in for chunkkv.runtime,
src/chunkkv/runtime.py:1-132).

`ChunkReuseRuntime` serves policies P0 and P2-P4 (chunk reuse at any position),
`PrefixCacheRuntime` serves P1 (longest exact token prefix).  Constructors,
`prefill(req, extra_tokens, logits_from) -> Outcome`, the placements and blend
settings handed to the engine, the gate calls, and the entries written back to the
store follow the reference step for step (runtime.py:50-93 and 117-132).  What
changes is the host work per request, which is O(segments) Python over buffers that
are built once:

- the request's tokens become one little-endian uint32 buffer; the hash of the
  tokens before each segment (the gate's exact-prefix test and the stored entry's
  `prefix_hash`, keys.py:15-20) is sha256 over a slice of that buffer, computed
  once per segment instead of twice from Python lists;
- each segment's lookup key is hashed once for the lookup and the write-back;
- the trust floor before each segment (types.py:48-51) comes from one running
  minimum over the segments, not a scan of all segments per call;
- the prefix cache keeps every served sequence's K/V in a paged HBM pool (one
  launch per request) and finds the longest common prefix with numpy compares
  over the stored token arrays instead of a Python loop over every stored token;
  a hit is served straight from the pages (PagedChunkKV.prefix, no copy).
"""

from __future__ import annotations

import hashlib
from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np

from chunkkv_b200.engine.base import BlendConfig, Placement, PrefillResult
from chunkkv_b200.store.keys import LookupKey, token_hash
from chunkkv_b200.store.kvstore import Entry, KVStore
from chunkkv_b200.store.pages import PAGE_TOKENS, PagePool, chunk_shape, write_chunk
from chunkkv_b200.types import ChunkedRequest, GateAction, GateDecision, TrustLevel


@dataclass
class Outcome:
    result: PrefillResult
    decisions: list[GateDecision] = field(default_factory=list)

    @property
    def stats(self) -> dict:
        return self.result.stats


def _token_bytes(tokens) -> bytes:
    a = np.asarray(tokens, dtype=np.int64)
    if a.size and (a.min() < 0 or a.max() >= 1 << 32):
        raise OverflowError("token ids must fit in 4 unsigned bytes")
    return a.astype("<u4").tobytes()


class RequestHashes:
    """Prefix hashes and trust floors of one request, from one token buffer.

    `prefix_hash(p)` equals token_hash(req.tokens[:p]); `trust_floor(p)` equals
    req.context_trust_before(p).  Each distinct position is hashed once."""

    def __init__(self, req: ChunkedRequest):
        self._buf = memoryview(_token_bytes(req.tokens))
        self._hashes: dict[int, str] = {}
        segs = sorted(req.segments, key=lambda s: s.start)
        self._starts = np.asarray([s.start for s in segs], dtype=np.int64)
        # floor before the i-th start = min trust of segments 0..i-1 in start order
        trust = np.asarray([int(s.trust) for s in segs], dtype=np.int64)
        self._floors = np.minimum.accumulate(trust) if trust.size else trust

    def prefix_hash(self, p: int) -> str:
        h = self._hashes.get(p)
        if h is None:
            d = hashlib.sha256()
            d.update(int(p).to_bytes(4, "little"))
            d.update(self._buf[: 4 * p])
            h = self._hashes[p] = d.hexdigest()
        return h

    def trust_floor(self, p: int) -> TrustLevel:
        n = int(np.searchsorted(self._starts, p, side="left"))  # segments starting before p
        return TrustLevel(int(self._floors[n - 1])) if n else TrustLevel.SYSTEM


class ChunkReuseRuntime:
    """Policies P0 (`enabled=False`) and P2-P4 over one engine, store and gate."""

    def __init__(self, engine, model_id: str, store: KVStore, gate, provenance: bool = True,
                 enabled: bool = True):
        self.engine = engine
        self.model_id = model_id
        self.store = store
        self.gate = gate
        self.provenance = provenance
        self.enabled = enabled

    def _key(self, req: ChunkedRequest, tokens) -> LookupKey:
        return LookupKey.build(tokens, self.model_id, req.tenant_id if self.provenance else None)

    def _decide(self, req, seg, entries, hashes: RequestHashes):
        fast = getattr(self.gate, "decide_hashed", None)
        if fast is not None:
            return fast(req, seg, entries, hashes.prefix_hash(seg.start), hashes.trust_floor(seg.start))
        return self.gate.decide(req, seg, entries)  # a gate with the reference's interface only

    def prefill(self, req: ChunkedRequest, extra_tokens: list[int] | None = None,
                logits_from: int | None = None) -> Outcome:
        """Prefill the request (plus optional teacher-forced `extra_tokens`)."""
        tokens = req.tokens + (extra_tokens or [])
        placements: list[Placement] = []
        decisions: list[GateDecision] = []
        keys: dict[int, LookupKey] = {}
        hashes = RequestHashes(req) if self.enabled else None
        if self.enabled:
            for i, seg in enumerate(req.segments):
                if not seg.reusable:
                    continue
                keys[i] = key = self._key(req, seg.tokens)
                entries = self.store.get(key)
                if not entries:
                    continue
                d, entry = self._decide(req, seg, entries, hashes)
                decisions.append(d)
                if d.action is GateAction.RECOMPUTE or entry is None:
                    continue
                entry.hits += 1
                placements.append(Placement(entry.kv, seg.start, d.ratio, exact=d.action is GateAction.REUSE))

        cfg = self.gate.config
        naive = cfg.mode == "naive" or all(d.action is GateAction.REUSE for d in decisions)
        blend = BlendConfig(
            recompute_ratio=0.0,
            full_first_layer=not naive,
            escalate_threshold=cfg.escalate_threshold if cfg.mode == "gated" else None,
        )
        result = self.engine.prefill(tokens, placements, blend, logits_from)

        if self.enabled:
            for i, seg in enumerate(req.segments):
                if seg.reusable:
                    entry = Entry(
                        kv=result.chunk(seg.start, seg.end),
                        context_id=req.context_id,
                        prefix_hash=hashes.prefix_hash(seg.start),
                        context_trust=hashes.trust_floor(seg.start),
                    )
                    self.store.put(keys[i], entry)
        return Outcome(result, decisions)


class PrefixCacheRuntime:
    """Policy P1: longest exact token prefix over previously prefilled requests.

    Like the reference (runtime.py:96-132): the sequences are kept in arrival order
    under a byte budget counted from their full per-layer K/V, the oldest dropped
    first (the newest is always kept); the longest common prefix with any kept
    sequence, capped at the last position whose logits are needed, is served as an
    exact placement at position 0; ties go to the earliest kept sequence.  Here each
    kept sequence is a PagedChunkKV in a page pool on the engine's device (created at
    the first request with room for `budget_bytes`, unless `pool` is given)."""

    def __init__(self, engine, budget_bytes: int = 4 << 30, pool: PagePool | None = None):
        self.engine = engine
        self.budget = budget_bytes
        self.pool = pool
        self._seqs: OrderedDict[int, tuple[np.ndarray, object]] = OrderedDict()
        self._next = 0
        self.bytes = 0

    def _lcp(self, toks: np.ndarray) -> tuple[int, object | None]:
        best, best_kv = 0, None
        for seq, kv in self._seqs.values():
            m = min(seq.size, toks.size)
            if m <= best:  # cannot be strictly longer
                continue
            diff = np.flatnonzero(seq[:m] != toks[:m])
            n = int(diff[0]) if diff.size else m
            if n > best:
                best, best_kv = n, kv
        return best, best_kv

    def _pool_for(self, kv) -> PagePool:
        L, H, D = chunk_shape(kv)
        if self.pool is None:
            per = PagePool.page_bytes_for(L, H, D)
            dev = getattr(self.engine, "device", "cuda")
            # the budget plus the newest sequence (always kept) and the partial last pages
            self.pool = PagePool.for_bytes(L, H, D, self.budget + self.budget // 8 + 64 * per, device=dev)
        elif not self.pool.matches(L, H, D):
            raise ValueError("sequence shape does not match the runtime's page pool")
        return self.pool

    def _drop_oldest(self) -> None:
        _, (_, kv) = self._seqs.popitem(last=False)
        self.bytes -= kv.nbytes
        self.pool.release(kv.page_ids)
        kv.revoke()

    def _keep(self, toks: np.ndarray, result: PrefillResult) -> None:
        whole = result.chunk(0, toks.size)
        pool = self._pool_for(whole)
        need = (toks.size + PAGE_TOKENS - 1) // PAGE_TOKENS
        if need > pool.n_pages:
            raise ValueError(f"sequence of {toks.size} tokens does not fit the page pool")
        ids = pool.alloc(need)
        while ids is None and self._seqs:
            self._drop_oldest()  # earlier gathers from these pages are ahead on the stream
            ids = pool.alloc(need)
        if ids is None:
            raise MemoryError("page pool exhausted")
        kv = write_chunk(pool, whole, ids)
        self._seqs[self._next] = (toks, kv)
        self._next += 1
        self.bytes += kv.nbytes
        while self.bytes > self.budget and len(self._seqs) > 1:
            self._drop_oldest()

    def prefill(self, req: ChunkedRequest, extra_tokens: list[int] | None = None,
                logits_from: int | None = None) -> Outcome:
        tokens = req.tokens + (extra_tokens or [])
        toks = np.frombuffer(_token_bytes(tokens), dtype="<u4")
        limit = (len(tokens) - 1) if logits_from is None else logits_from
        n, kv = self._lcp(toks)
        n = min(n, limit)
        placements = [Placement(kv.prefix(n), 0, exact=True)] if kv is not None and n > 0 else []
        result = self.engine.prefill(tokens, placements, BlendConfig(full_first_layer=False), logits_from)
        self._keep(toks, result)
        return Outcome(result)


__all__ = ["ChunkReuseRuntime", "Outcome", "PrefixCacheRuntime", "RequestHashes", "token_hash"]
