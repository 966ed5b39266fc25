"""Paged HBM pool for cached chunk K/V.

One device tensor holds every page:
    pages[n_pages][n_layers][2 (K, V)][n_kv_heads][16 tokens][head_dim]  bf16
so a page is 16 tokens of one chunk across all layers, and each
(layer, K|V, head) piece of a page is 16*head_dim contiguous values — the unit
the gather/scatter kernels stream.  A chunk is a list of page ids plus its
length and the position it was computed at (PagedChunkKV).  Free pages are a
host-side stack; allocation and release never touch the device.
"""

from __future__ import annotations

import numpy as np
import torch

from chunkkv_b200 import ops
from chunkkv_b200.engine.staging import Staging, pack_upload

PAGE_TOKENS = ops.PAGE_TOKENS


class PagePool:
    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, n_pages: int, device="cuda"):
        if n_pages <= 0:
            raise ValueError("page pool needs at least one page")
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        self.pages = torch.empty((n_pages, n_layers, 2, n_kv_heads, PAGE_TOKENS, head_dim),
                                 dtype=torch.bfloat16, device=device)
        self._free = list(range(n_pages - 1, -1, -1))
        self._stage = Staging(slots=64)  # page-pointer uploads, one slot per write in flight

    @classmethod
    def for_bytes(cls, n_layers, n_kv_heads, head_dim, nbytes: int, device="cuda") -> "PagePool":
        per = cls.page_bytes_for(n_layers, n_kv_heads, head_dim)
        return cls(n_layers, n_kv_heads, head_dim, max(1, nbytes // per), device)

    @staticmethod
    def page_bytes_for(n_layers, n_kv_heads, head_dim) -> int:
        return n_layers * 2 * n_kv_heads * PAGE_TOKENS * head_dim * 2

    @property
    def n_pages(self) -> int:
        return self.pages.shape[0]

    @property
    def page_bytes(self) -> int:
        return self.page_bytes_for(self.n_layers, self.n_kv_heads, self.head_dim)

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def alloc(self, n: int) -> np.ndarray | None:
        if n > len(self._free):
            return None
        ids = [self._free.pop() for _ in range(n)]
        return np.asarray(ids, dtype=np.int32)

    def release(self, ids: np.ndarray) -> None:
        self._free.extend(int(i) for i in ids[::-1])

    def matches(self, n_layers, n_kv_heads, head_dim) -> bool:
        return (n_layers, n_kv_heads, head_dim) == (self.n_layers, self.n_kv_heads, self.head_dim)

    def write(self, page_ids: np.ndarray, length: int, keys: list[torch.Tensor],
              values: list[torch.Tensor]) -> None:
        """Scatter per-layer (1|H, H, len, D)-shaped K/V into the pages (one launch)."""
        dev = self.pages.device
        ks = [_as_source(k, dev) for k in keys]
        vs = [_as_source(v, dev) for v in values]
        stride = ks[0].stride(-3)
        if any(t.stride(-3) != stride for t in ks + vs):
            ks = [k.contiguous() for k in ks]
            vs = [v.contiguous() for v in vs]
            stride = ks[0].stride(-3)
        d, _ = pack_upload([("kp", np.asarray([k.data_ptr() for k in ks], dtype=np.uint64)),
                            ("vp", np.asarray([v.data_ptr() for v in vs], dtype=np.uint64)),
                            ("ids", np.asarray(page_ids, dtype=np.int32))], self._stage, dev)
        ops.pages_write(self.pages, d["ids"], length, d["kp"], d["vp"], stride)
        # No host sync: device temporaries made by _as_source are freed into torch's
        # stream-ordered allocator, so no later work on this stream can reuse them
        # before the copy has run.


def _as_source(t: torch.Tensor, dev) -> torch.Tensor:
    if t.dim() == 4:
        t = t[0]
    ok = (t.is_cuda and t.device == dev and t.dtype == torch.bfloat16 and t.stride(-1) == 1
          and t.stride(-2) == t.shape[-1] and t.data_ptr() % 16 == 0 and t.stride(-3) % 8 == 0)
    return t if ok else t.to(device=dev, dtype=torch.bfloat16).contiguous()


class _LayerList:
    """`chunk.keys` / `chunk.values` of a paged chunk: layer li materialises (1, H, len, D)."""

    def __init__(self, chunk: "PagedChunkKV", kv: int):
        self._c, self._kv = chunk, kv

    def __len__(self) -> int:
        return self._c.pool.n_layers

    def __getitem__(self, li: int) -> torch.Tensor:
        n = len(self)
        if li < 0:
            li += n
        if not 0 <= li < n:
            raise IndexError(li)
        k, v = self._c.materialize(li, li + 1)
        return (k if self._kv == 0 else v)[0].unsqueeze(0)

    def __iter__(self):
        return (self[i] for i in range(len(self)))


class _Lease:
    """Shared by a stored chunk and every view made from it (``prefix``); cleared when the
    owner (a KVStore or the prefix cache) gives the pages back to the pool."""

    __slots__ = ("alive",)

    def __init__(self):
        self.alive = True


class PagedChunkKV:
    """ChunkKV-compatible view of a chunk stored in a PagePool.

    Unlike the reference's per-layer tensors, which stay valid after their store entry is
    evicted, a paged chunk's pages go back to the pool on eviction and may then be
    rewritten with another chunk.  Eviction therefore revokes the chunk: reading its K/V
    afterwards (``keys``/``values``, ``materialize``, ``prefix``, or a prefill placement)
    raises ValueError instead of returning another chunk's data.  ``length``, ``start``
    and ``nbytes`` stay readable."""

    def __init__(self, pool: PagePool, page_ids: np.ndarray, length: int, start: int, src_offset: int = 0,
                 lease: _Lease | None = None):
        self.pool, self.page_ids, self.start = pool, np.asarray(page_ids, np.int32), int(start)
        self._length, self.src_offset = int(length), int(src_offset)
        self._lease = _Lease() if lease is None else lease

    @property
    def alive(self) -> bool:
        """False once the owner has evicted the chunk and released its pages."""
        return self._lease.alive

    def revoke(self) -> None:
        """Mark the chunk (and every view sharing its pages) as evicted."""
        self._lease.alive = False

    def check_alive(self) -> None:
        if not self._lease.alive:
            raise ValueError("this chunk was evicted from its store; its pages may now hold another chunk")

    @property
    def length(self) -> int:
        return self._length

    @property
    def keys(self) -> _LayerList:
        return _LayerList(self, 0)

    @property
    def values(self) -> _LayerList:
        return _LayerList(self, 1)

    @property
    def nbytes(self) -> int:
        """Bytes of the K/V it holds, counted like the reference's per-layer tensors."""
        p = self.pool
        return p.n_layers * 2 * p.n_kv_heads * self._length * p.head_dim * 2

    def prefix(self, n: int) -> "PagedChunkKV":
        """The chunk's first `n` tokens: the same pages, no copy."""
        self.check_alive()
        if not 0 <= n <= self._length:
            raise ValueError(f"prefix of {n} tokens from a chunk of {self._length}")
        pages = (self.src_offset + n + PAGE_TOKENS - 1) // PAGE_TOKENS
        return PagedChunkKV(self.pool, self.page_ids[:pages], n, self.start, self.src_offset, self._lease)

    def materialize(self, layer_lo: int = 0, layer_hi: int | None = None):
        """Dense copies [layers, H, len, D] of K and V (as stored, no shift)."""
        self.check_alive()
        p = self.pool
        layer_hi = p.n_layers if layer_hi is None else layer_hi
        dev = p.pages.device
        n_l = layer_hi - layer_lo
        k = torch.empty((n_l, p.n_kv_heads, self._length, p.head_dim), dtype=torch.bfloat16, device=dev)
        v = torch.empty_like(k)
        meta = torch.tensor([[0, self._length, 0, 0, layer_lo, layer_hi, self.src_offset, 0]],
                            dtype=torch.int32).to(dev)
        table = torch.from_numpy(self.page_ids).to(dev)
        inv = torch.zeros(p.head_dim // 2, dtype=torch.float32, device=dev)  # unused at delta 0
        ops.blend_gather_paged(p.pages, table, meta, inv, k, v, layer_lo, layer_hi)
        return k, v


def chunk_shape(kv) -> tuple[int, int, int]:
    """(layers, KV heads, head_dim) of a chunk given as per-layer tensors or a cache view."""
    from chunkkv_b200.engine.base import CacheChunkKV

    if isinstance(kv, CacheChunkKV) and kv.viewable:
        L, k0 = kv.n_layers, kv.view(0, 0)
    else:
        L, k0 = len(kv.keys), kv.keys[0]
    return L, k0.shape[-3], k0.shape[-1]


def write_chunk(pool: PagePool, kv, page_ids: np.ndarray) -> PagedChunkKV:
    """Copy a chunk's K/V into `page_ids` of the pool (one launch) and return the paged
    view.  A cache view of an engine result (CacheChunkKV) is read in place, without
    the per-layer copies."""
    from chunkkv_b200.engine.base import CacheChunkKV

    length = kv.length
    if isinstance(kv, CacheChunkKV) and kv.viewable:
        L = pool.n_layers
        pool.write(page_ids, length, [kv.view(li, 0) for li in range(L)], [kv.view(li, 1) for li in range(L)])
    else:
        pool.write(page_ids, length, list(kv.keys), list(kv.values))
    return PagedChunkKV(pool, page_ids, length, kv.start)
