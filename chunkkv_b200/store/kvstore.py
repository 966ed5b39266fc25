"""Chunk K/V store over a paged HBM pool (drop-in for chunkkv.store.kvstore).

Bookkeeping follows src/chunkkv/store/kvstore.py:20-63: LRU order by key, a
byte budget counted from the entries' K/V sizes, at most `max_variants`
entries per key (oldest dropped), and an entry whose (prefix_hash,
context_trust) is already stored is not stored again.  The K/V itself lives
in one PagePool on the device: `put` copies an entry's per-layer tensors into
pages with one kernel launch and swaps `entry.kv` for a PagedChunkKV view that
the engine gathers from directly.  An evicted entry's pages go back to the pool
and its PagedChunkKV is revoked (reading it raises ValueError), where the
reference's evicted tensors would stay readable.  The pool is created at the first put
(shapes taken from that entry) unless one is passed in; when it runs out of
pages, least-recently-used keys are evicted as for the byte budget.
"""

from __future__ import annotations

import itertools
from collections import OrderedDict
from dataclasses import dataclass, field

from chunkkv_b200.engine.base import CacheChunkKV
from chunkkv_b200.store.keys import LookupKey
from chunkkv_b200.store.pages import PAGE_TOKENS, PagedChunkKV, PagePool, chunk_shape, write_chunk
from chunkkv_b200.types import TrustLevel

_ids = itertools.count()


def entry_bytes(entry) -> int:
    """K/V bytes of an entry, counted like the reference (kvstore.py:29-31) but without
    reading paged K/V back; works for this module's Entry and the reference's."""
    kv = entry.kv
    if isinstance(kv, PagedChunkKV):
        return kv.nbytes
    return sum(k.nbytes + v.nbytes for k, v in zip(kv.keys, kv.values))


@dataclass
class Entry:
    kv: object  # ChunkKV (per-layer tensors) until stored, then PagedChunkKV
    context_id: str
    prefix_hash: str
    context_trust: TrustLevel
    id: str = field(default_factory=lambda: f"e{next(_ids)}")
    hits: int = 0

    @property
    def nbytes(self) -> int:
        return entry_bytes(self)


class KVStore:
    def __init__(self, budget_bytes: int = 4 << 30, max_variants: int = 4, pool: PagePool | None = None,
                 pool_bytes: int | None = None, device=None):
        self.budget = budget_bytes
        self.max_variants = max_variants
        self._data: OrderedDict[LookupKey, list[Entry]] = OrderedDict()
        self.bytes = 0
        self.pool = pool
        self._pool_bytes = pool_bytes
        self._device = device

    # -- reference API --------------------------------------------------------
    def get(self, key: LookupKey) -> list[Entry]:
        entries = self._data.get(key)
        if entries:
            self._data.move_to_end(key)
        return list(entries or [])

    def put(self, key: LookupKey, entry: Entry) -> None:
        entries = self._data.setdefault(key, [])
        if any(e.prefix_hash == entry.prefix_hash and e.context_trust == entry.context_trust for e in entries):
            self._data.move_to_end(key)
            return
        try:
            self._store_pages(entry, protect=key)
        except BaseException:
            if not self._data.get(key):  # no key left behind without entries
                self._data.pop(key, None)
            raise
        entries = self._data.setdefault(key, entries)
        entries.append(entry)
        self.bytes += entry_bytes(entry)
        while len(entries) > self.max_variants:
            self._drop(entries.pop(0))
        self._data.move_to_end(key)
        self._evict()

    def __len__(self) -> int:
        return sum(len(v) for v in self._data.values())

    # -- paging ------------------------------------------------------------------
    def _ensure_pool(self, kv) -> PagePool:
        L, H, D = chunk_shape(kv)
        if self.pool is None:
            nbytes = self._pool_bytes or (self.budget + self.budget // 8)
            k0 = kv.view(0, 0) if isinstance(kv, CacheChunkKV) and kv.viewable else kv.keys[0]
            dev = self._device or (k0.device if getattr(k0, "is_cuda", False) else "cuda")
            self.pool = PagePool.for_bytes(L, H, D, nbytes, device=dev)
        elif not self.pool.matches(L, H, D):
            raise ValueError("entry shape does not match the store's page pool")
        return self.pool

    def _store_pages(self, entry: Entry, protect: LookupKey) -> None:
        kv = entry.kv
        if isinstance(kv, PagedChunkKV):
            return
        pool = self._ensure_pool(kv)
        need = (kv.length + PAGE_TOKENS - 1) // PAGE_TOKENS
        if need > pool.n_pages:
            raise ValueError(f"chunk of {kv.length} tokens does not fit the page pool")
        ids = pool.alloc(need)
        while ids is None:
            if not self._evict_one(protect):
                raise MemoryError("page pool exhausted")
            ids = pool.alloc(need)
        entry.kv = write_chunk(pool, kv, ids)

    def _drop(self, e: Entry) -> None:
        self.bytes -= entry_bytes(e)
        if isinstance(e.kv, PagedChunkKV) and e.kv.pool is self.pool:
            self.pool.release(e.kv.page_ids)
            e.kv.revoke()  # the pages may be rewritten: reading this entry's K/V now raises

    def _evict_one(self, protect: LookupKey | None = None) -> bool:
        for key in self._data:
            if key == protect:
                continue
            entries = self._data.pop(key)
            for e in entries:
                self._drop(e)
            return True
        return False

    def _evict(self) -> None:
        while self.bytes > self.budget and self._data:
            _, entries = self._data.popitem(last=False)
            for e in entries:
                self._drop(e)
