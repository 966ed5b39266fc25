"""Seeded blend-prefill scenarios shared by the golden-fixture generator and the tests.

A scenario is: one or more "first" prefills whose K/V provide the cached chunks,
then one blend request that places those chunks at new offsets.  Token ids are
uniform random from `random.Random(seed)`; weights come from
chunkkv_b200.engine.weights.random_state_dict(shape, seed) in bf16.
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field


@dataclass(frozen=True)
class Scenario:
    name: str
    shape: str
    dtype: str                 # "fp32" or "bf16": the reference model dtype
    n_chunks: int
    chunk_len: int
    prefix_len: int
    query_len: int
    ratio: float = 0.15
    n_sink: int = 4
    escalate: float | None = None
    exact_first: bool = False   # first chunk served exact at its original offset (no prefix)
    first_ratio: float | None = None  # per-placement ratio of the moved chunks (None = config)
    full_first_layer: bool = True
    seed: int = 0
    store_full_logits: bool = True


SCENARIOS = {
    # GQA 2:1, head_dim 64, fp32: the main pin of the oracle
    "tiny_fp32": Scenario("tiny_fp32", "tiny", "fp32", n_chunks=3, chunk_len=48, prefix_len=16,
                          query_len=16, ratio=0.3),
    # same, bf16 reference model (rounding points of a bf16 deployment)
    "tiny_bf16": Scenario("tiny_bf16", "tiny", "bf16", n_chunks=3, chunk_len=48, prefix_len=16,
                          query_len=16, ratio=0.3, seed=1),
    # escalation probe armed low enough that chunks escalate
    "tiny_escalate": Scenario("tiny_escalate", "tiny", "fp32", n_chunks=4, chunk_len=40,
                              prefix_len=8, query_len=8, ratio=0.25, escalate=3e-4, seed=2),
    # leading exact chunk + ratio 1.0 moved chunk (test_mlx_engine.py:86-99 regression shape)
    "tiny_exact_overflow": Scenario("tiny_exact_overflow", "tiny", "fp32", n_chunks=2, chunk_len=40,
                                    prefix_len=0, query_len=12, exact_first=True, first_ratio=1.0,
                                    seed=3),
    # GQA 7:1 at head_dim 128 (the 7B head layout)
    "tiny7_fp32": Scenario("tiny7_fp32", "tiny7", "fp32", n_chunks=4, chunk_len=64, prefix_len=16,
                           query_len=16, ratio=0.15, seed=4),
    # Qwen2.5-0.5B shape, 4 x 256 chunks cached at 0..1023, served in a
    # seeded permutation behind a 32-token prefix plus a 64-token query, 15 % + 4 sinks
    "cfg1_0p5b": Scenario("cfg1_0p5b", "qwen2.5-0.5b", "fp32", n_chunks=4, chunk_len=256,
                          prefix_len=32, query_len=64, ratio=0.15, n_sink=4, store_full_logits=False),
}


@dataclass
class Built:
    first_tokens: list[list[int]]            # token lists of the first prefills
    chunk_src: list[tuple[int, int]]         # per chunk: (first-prefill index, start in it)
    tokens: list[int]                        # the blend request
    place: list[dict] = field(default_factory=list)  # chunk, start, ratio, exact


def build(sc: Scenario, vocab: int) -> Built:
    rng = random.Random(sc.seed)
    rand = lambda n: [rng.randrange(vocab) for _ in range(n)]  # noqa: E731
    chunks = [rand(sc.chunk_len) for _ in range(sc.n_chunks)]
    prefix, query = rand(sc.prefix_len), rand(sc.query_len)
    if sc.exact_first:
        # chunk 0 first at offset 0 (with whatever follows), chunk 1.. computed after another prefix
        other = rand(7)
        first = [chunks[0] + query, other + sum(chunks[1:], [])]
        src = [(0, 0)] + [(1, len(other) + i * sc.chunk_len) for i in range(sc.n_chunks - 1)]
        tokens = chunks[0] + sum(chunks[1:], []) + query
        place = [dict(chunk=0, start=0, ratio=None, exact=True)]
        for i in range(1, sc.n_chunks):
            place.append(dict(chunk=i, start=i * sc.chunk_len, ratio=sc.first_ratio, exact=False))
        return Built(first, src, tokens, place)
    first = [sum(chunks, [])]
    src = [(0, i * sc.chunk_len) for i in range(sc.n_chunks)]
    order = list(range(sc.n_chunks))
    while order == sorted(order) and sc.n_chunks > 1:
        rng.shuffle(order)
    tokens = list(prefix)
    place = []
    for c in order:
        place.append(dict(chunk=c, start=len(tokens), ratio=sc.first_ratio, exact=False))
        tokens += chunks[c]
    tokens += query
    return Built(first, src, tokens, place)
