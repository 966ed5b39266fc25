"""Cache keys (drop-in for chunkkv.store.keys, src/chunkkv/store/keys.py:15-31).

The lookup key is content + model (+ tenant when provenance is on).  The content
hash is sha256 over the token count and the tokens, each as 4 little-endian
bytes — the same digest as the reference, computed from one numpy buffer
instead of a Python loop.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np


def token_hash(tokens) -> str:
    a = np.asarray(tokens, dtype=np.int64)
    if a.size and (a.min() < 0 or a.max() >= 1 << 32):
        raise OverflowError("token ids must fit in 4 unsigned bytes")
    h = hashlib.sha256()
    h.update(int(a.size).to_bytes(4, "little"))
    h.update(a.astype("<u4").tobytes())
    return h.hexdigest()


@dataclass(frozen=True)
class LookupKey:
    content: str
    model_id: str
    tenant_id: str | None  # None when provenance keys are off (P2/P3)

    @classmethod
    def build(cls, tokens, model_id: str, tenant_id: str | None) -> "LookupKey":
        return cls(token_hash(tokens), model_id, tenant_id)
