"""Runtime, gate and policy bookkeeping against the reference's own runtimes.

tests/golden/runtime_policies.json was produced by make_runtime_golden.py, which
ran the reference's bench/policies.py P0-P4 runtimes (runtime.py, gate.py,
kvstore.py) over the request stream of runtime_stream.py with a stand-in engine.
The same stream goes through this package's runtimes here, with a stand-in engine
and a host-only page pool, and every engine call (tokens, placements, blend
settings), every gate decision and the final store state must be the same.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

from runtime_stream import CHUNK_BUDGET, PREFIX_BUDGET, build_request, stream  # noqa: E402

from chunkkv_b200 import types  # noqa: E402
from chunkkv_b200.engine.base import PrefillResult  # noqa: E402


class HostPool:
    """Page bookkeeping without device memory (PagePool's host-side interface)."""

    n_layers, n_kv_heads, head_dim = 2, 1, 8

    def __init__(self, n_pages: int = 1 << 16):
        self._free = list(range(n_pages - 1, -1, -1))
        self.n_pages = n_pages

    def matches(self, L, H, D):
        return (L, H, D) == (self.n_layers, self.n_kv_heads, self.head_dim)

    def alloc(self, n):
        if n > len(self._free):
            return None
        return np.asarray([self._free.pop() for _ in range(n)], dtype=np.int32)

    def release(self, ids):
        self._free.extend(int(i) for i in ids[::-1])

    def write(self, ids, length, keys, values):
        assert len(keys) == len(values) == self.n_layers and keys[0].shape[-2] == length


class Engine:
    def __init__(self):
        self.calls = []

    def prefill(self, tokens, placements=None, config=None, logits_from=None):
        self.chunks = [p.chunk for p in placements or []]
        self.calls.append({
            "n": len(tokens), "logits_from": logits_from,
            "placements": [[p.start, p.ratio, bool(p.exact), p.chunk.start, p.chunk.length]
                           for p in placements or []],
            "blend": [config.recompute_ratio, config.full_first_layer, config.escalate_threshold],
        })
        k = [torch.zeros((1, 1, len(tokens), 8), dtype=torch.bfloat16) for _ in range(2)]
        return PrefillResult(None, None, k, [t.clone() for t in k], {}, copy=lambda a: a.clone())


def _golden():
    return json.loads((GOLDEN / "runtime_policies.json").read_text())


@pytest.mark.parametrize("policy", ["P0", "P1", "P2", "P3", "P4"])
def test_policy_runtime_matches_reference(policy):
    from chunkkv_b200.policies import build
    from chunkkv_b200.store.kvstore import KVStore

    ref = _golden()["policies"][policy]
    eng = Engine()
    budget = PREFIX_BUDGET if policy == "P1" else CHUNK_BUDGET
    rt = build(policy, eng, "m", budget_bytes=budget, ratio=0.15, store=KVStore(budget, pool=HostPool()))
    if policy == "P1":
        rt.pool = HostPool()
    decisions = []
    for r in stream(_golden()["stream_seed"]):
        o = rt.prefill(build_request(r, types))
        decisions.append([[d.segment, d.action.value, d.reason, d.ratio] for d in o.decisions])
    assert eng.calls == ref["calls"]
    assert decisions == ref["decisions"]
    if policy == "P1":
        assert [len(seq) for seq, _ in rt._seqs.values()] == ref["kept"]
        assert rt.bytes == ref["bytes"]
    else:
        store = [[[e.context_id, e.prefix_hash, int(e.context_trust), e.hits, e.kv.start, e.kv.length]
                  for e in entries] for entries in rt.store._data.values()]
        assert store == ref["store"]
        assert rt.store.bytes == ref["bytes"]


def test_request_hashes_match_token_hash_and_trust_floor():
    from chunkkv_b200.runtime import RequestHashes
    from chunkkv_b200.store.keys import token_hash

    for r in stream(3, n_requests=6):
        req = build_request(r, types)
        h = RequestHashes(req)
        for p in sorted({s.start for s in req.segments} | {0, len(req.tokens)}):
            assert h.prefix_hash(p) == token_hash(req.tokens[:p])
            assert h.trust_floor(p) == req.context_trust_before(p)


def test_gate_with_reference_interface_is_used_as_is():
    """A gate that only has decide() (the reference's interface) still drives the runtime."""
    from chunkkv_b200.gate import GateConfig, ReuseGate
    from chunkkv_b200.runtime import ChunkReuseRuntime
    from chunkkv_b200.store.kvstore import KVStore

    class PlainGate:
        def __init__(self):
            self._g = ReuseGate(GateConfig(ratio_same_context=0.15, ratio_other_context=0.3,
                                           escalate_threshold=None))  # as policies.build("P4")
            self.config = self._g.config
            self.calls = 0

        def decide(self, req, seg, entries):
            self.calls += 1
            return self._g.decide(req, seg, entries)

    ref = _golden()["policies"]["P4"]
    eng, gate = Engine(), PlainGate()
    rt = ChunkReuseRuntime(eng, "m", KVStore(CHUNK_BUDGET, pool=HostPool()), gate, provenance=True)
    for r in stream(_golden()["stream_seed"]):
        rt.prefill(build_request(r, types))
    assert eng.calls == ref["calls"] and gate.calls == sum(len(d) for d in ref["decisions"])


def test_prefix_cache_lcp_ties_and_limit():
    """Longest common prefix: the earliest kept sequence wins a tie, the match is
    capped below the last position (its logits are needed) or at logits_from."""
    from chunkkv_b200.runtime import PrefixCacheRuntime

    eng = Engine()
    rt = PrefixCacheRuntime(eng, budget_bytes=1 << 30, pool=HostPool())

    def req(tokens):
        return types.ChunkedRequest(tokens, [types.Segment(0, "user", types.TrustLevel.USER, 0, tokens, False)],
                                    "t", "c")

    rt.prefill(req([1, 2, 3, 4, 5]))
    rt.prefill(req([1, 2, 3, 9]))
    rt.prefill(req([1, 2, 3, 4, 5]))      # whole match, capped at n - 1 = 4
    assert eng.calls[-1]["placements"] == [[0, None, True, 0, 4]]
    first_pages = next(iter(rt._seqs.values()))[1].page_ids
    rt.prefill(req([1, 2, 3, 7, 7]))      # ties (3 tokens) with all three kept sequences
    assert eng.calls[-1]["placements"] == [[0, None, True, 0, 3]]
    assert np.array_equal(eng.chunks[0].page_ids, first_pages[:1])  # the earliest one serves
    rt.prefill(req([1, 2, 3, 4, 5, 6]), logits_from=2)
    assert eng.calls[-1]["placements"] == [[0, None, True, 0, 2]]
    rt.prefill(req([8, 8]))
    assert eng.calls[-1]["placements"] == []


def test_report_summary_matches_reference():
    """harness.summarize / boot_ci against the reference's bench/report.py outputs
    (tests/golden/make_report_golden.py)."""
    from chunkkv_b200.harness import boot_ci, summarize

    g = json.loads((GOLDEN / "report_summary.json").read_text())
    # fields the reference derives from labelled real-text traces (accuracy, attacks,
    # conflicting contexts); synthetic replays have no labels, so they are not summarised
    label_fields = {"acc", "acc_ci", "attack_success", "match_p0_conflict"}
    for case in g["cases"]:
        got = json.loads(json.dumps(summarize(case["rows"], case["skip_first"])))
        want = case["summary"]
        assert set(want) - set(got) <= label_fields and set(got) <= set(want)
        assert got == {k: v for k, v in want.items() if k in got}
    assert list(boot_ci(np.asarray(g["boot"]["x"], dtype=float))) == g["boot"]["ci"]
    # the one-matrix resampling equals one draw per resample, at any sample size
    for n in (1, 2, 5, 23, 37, 64):
        x = np.random.default_rng(n).random(n)
        rng = np.random.default_rng(0)
        per = [np.mean(x[rng.integers(0, n, n)]) for _ in range(2000)]
        assert boot_ci(x) == (float(np.percentile(per, 2.5)), float(np.percentile(per, 97.5)))


def test_compare_to_p0():
    from chunkkv_b200.harness import compare_to_p0

    lp0 = np.log(np.array([0.5, 0.25, 0.25]))
    lp = np.log(np.array([0.25, 0.5, 0.25]))
    c = compare_to_p0(lp, [1, 2, 3, 9], lp0, [1, 2, 4, 9])
    assert abs(c["kl"] - 0.25 * np.log(2)) < 1e-12
    assert c["match_p0"] is False and c["agree_prefix"] == 0.5
    assert compare_to_p0(lp0, [5], lp0, [5]) == {"kl": 0.0, "match_p0": True, "agree_prefix": 1.0}
