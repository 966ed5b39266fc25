"""A seeded multi-tenant request stream for the runtime and policy fixtures.

Each request is plain data: tenant, context id and a list of segments
(role, trust, tokens, reusable).  System prompts are SYSTEM, documents and tool
outputs TOOL, user turns USER (never reusable).  Documents come back in other
orders, after other prefixes, under other contexts and tenants, and after user
turns, so every gate rule fires: exact prefix, same context, other context, and
the trust floor.
"""

from __future__ import annotations

import random

SYSTEM, TOOL, USER = 2, 1, 0


def stream(seed: int = 0, n_requests: int = 18) -> list[dict]:
    rng = random.Random(seed)

    def toks(n):
        return [rng.randrange(1, 5000) for _ in range(n)]

    systems = {"ctxA": toks(40), "ctxB": toks(36)}
    docs = [toks(rng.randrange(24, 72)) for _ in range(6)]
    reqs = []
    for i in range(n_requests):
        tenant = "t0" if i % 3 else "t1"
        ctx = "ctxA" if rng.random() < 0.6 else "ctxB"
        segs = [("system", SYSTEM, systems[ctx], True)]
        if rng.random() < 0.3:  # a user turn before the documents lowers the trust floor
            segs.append(("user", USER, toks(12), False))
        picks = rng.sample(range(len(docs)), rng.randrange(2, 5))
        if i >= 2 and rng.random() < 0.35:  # repeat an earlier request's document order
            picks = reqs[rng.randrange(i)]["picks"]
        for d in picks:
            segs.append(("tool", TOOL, docs[d], True))
        segs.append(("user", USER, toks(rng.randrange(8, 20)), False))
        reqs.append({"tenant": tenant, "context": ctx, "segments": segs, "picks": list(picks)})
    return reqs


def build_request(r: dict, types):
    """ChunkedRequest of module `types` (the reference's chunkkv.types or chunkkv_b200.types)."""
    segs, tokens = [], []
    for i, (role, trust, t, reusable) in enumerate(r["segments"]):
        segs.append(types.Segment(i, role, types.TrustLevel(trust), len(tokens), list(t), reusable))
        tokens += t
    return types.ChunkedRequest(tokens, segs, r["tenant"], r["context"])


# budgets (bytes) small enough that the stores evict during the stream; the fake
# engine's K/V is 2 layers x 1 head x 8 dims of bf16, 64 bytes per token
BYTES_PER_TOKEN = 2 * 2 * 1 * 8 * 2
CHUNK_BUDGET = 900 * BYTES_PER_TOKEN
PREFIX_BUDGET = 700 * BYTES_PER_TOKEN
