"""Host-side logic that needs no GPU: the C ABI library, planning, keys, store
bookkeeping, weight packing, and the refusal of CPU tensors (no CPU fallback)."""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest
import torch

from chunkkv_b200 import _lib, ops
from chunkkv_b200.engine.base import BlendConfig, ChunkKV, Placement, plan_arrays, plan_positions
from chunkkv_b200.engine.weights import SHAPES, interleave_gate_up, param_shapes
from chunkkv_b200.store.keys import LookupKey, token_hash
from oracle.blend_oracle import plan_positions as ref_plan

ROOT = Path(__file__).resolve().parent.parent


def test_library_loads_and_exports_every_header_symbol():
    header = (ROOT / "include" / "chunkkv_b200.h").read_text()
    declared = set(re.findall(r"CKV_API\s+[\w\s\*]+?\b(ckv_\w+)\s*\(", header))
    assert len(declared) >= 20
    assert declared == set(_lib.SIGNATURES), declared ^ set(_lib.SIGNATURES)
    lib = _lib.load()
    for name in declared:
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.ckv_version()


def test_status_codes_map_to_reference_exceptions():
    # a null-pointer call is refused on the host before anything launches
    with pytest.raises(ValueError):
        _lib.call("ckv_rmsnorm", None, None, None, 1, 8, 1e-6, None)
    assert "null" in _lib.last_error()
    # hidden above the one-CTA-per-row limit is refused before any launch
    with pytest.raises(ValueError):
        _lib.call("ckv_rmsnorm", 16, 16, 16, 1, 5128, 1e-6, None)
    assert "5120" in _lib.last_error()
    with pytest.raises(NotImplementedError):
        _lib.call("ckv_attention", 16, 16, 16, 16, 16, 1, 1, 1, 96, 8, 1.0, None, 0, None)


def test_ops_refuse_cpu_tensors():
    x = torch.zeros((4, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.linear(x, x)
    with pytest.raises(ValueError, match="CUDA"):
        ops.rmsnorm(x, x[0], 1e-6)


class _C:
    def __init__(self, n):
        self.length = n


@pytest.mark.parametrize("seed", range(5))
def test_plan_arrays_matches_reference_plan(seed):
    rng = np.random.default_rng(seed)
    n = 300
    pl = []
    for _ in range(rng.integers(0, 6)):
        ln = int(rng.integers(1, 60))
        st = int(rng.integers(0, n - ln))
        pl.append(Placement(_C(ln), st, exact=bool(rng.integers(0, 2))))
    n_sink = int(rng.integers(0, 5))
    got = plan_arrays(n, pl, n_sink)
    ref = ref_plan(n, pl, n_sink)
    assert got.cached.tolist() == ref[0] and got.exact.tolist() == ref[1] and got.sink.tolist() == ref[2]
    assert plan_positions(n, pl, n_sink) == ref
    f = got.pos_flags()
    assert ((f & 1) == got.cached).all() and (((f >> 1) & 1) == got.sink).all() and ((f >> 2) == got.exact).all()


def test_plan_rejects_placement_past_the_request():
    with pytest.raises(IndexError):
        plan_arrays(10, [Placement(_C(8), 5)], 2)


# Known answers computed with the reference's chunkkv.store.keys.token_hash.
TOKEN_HASH_KAT = [
    ([], "df3f619804a92fdb4057192dc43dd748ea778adc52bc498ce80524c014b81119"),
    ([0], "7c9fa136d4413fa6173637e883b6998d32e1d675f88cddff9dcbcf331820f4b8"),
    ([1, 2, 3], "374d429ee174762e85d14ea494b50c91a44a1557227814f14650940d7e283790"),
    ([151935, 7, 42, 0, 65536], "ef433809cebf84ac5f48362a7f127ca7d01a48fda4fc79bd1008b89617ea1481"),
    (list(range(300)), "db9457e983ac73cbb3c2b9795a1c88168ae6964df3387c8e1f0086dbc4cce20b"),
]


@pytest.mark.parametrize("tokens,digest", TOKEN_HASH_KAT)
def test_token_hash_known_answers(tokens, digest):
    assert token_hash(tokens) == digest
    assert LookupKey.build(tokens, "m", None) == LookupKey(digest, "m", None)


def test_token_hash_rejects_negative_ids():
    with pytest.raises(OverflowError):
        token_hash([1, -2])


# ---- store bookkeeping (kvstore.py:47-63 semantics) over a fake page pool
class FakePool:
    n_layers, n_kv_heads, head_dim = 2, 1, 8

    def __init__(self):
        self.released = []

    def release(self, ids):
        self.released.extend(int(i) for i in ids)


def _entry(pool, n_tokens, prefix="p", trust=2, ctx="c"):
    from chunkkv_b200.store.kvstore import Entry
    from chunkkv_b200.store.pages import PagedChunkKV
    from chunkkv_b200.types import TrustLevel

    kv = PagedChunkKV(pool, np.arange((n_tokens + 15) // 16), n_tokens, 0)
    return Entry(kv, ctx, prefix, TrustLevel(trust))


def test_kvstore_lru_budget_variants_and_dedup():
    from chunkkv_b200.store.kvstore import KVStore

    pool = FakePool()
    per_tok = 2 * 2 * 1 * 8 * 2  # layers * (K,V) * heads * D * bf16
    st = KVStore(budget_bytes=3 * 100 * per_tok, max_variants=2, pool=pool)
    k = [LookupKey.build([i], "m", None) for i in range(5)]
    st.put(k[0], _entry(pool, 100))
    st.put(k[1], _entry(pool, 100))
    assert st.bytes == 200 * per_tok and len(st) == 2
    # same (prefix_hash, trust) is not stored twice
    st.put(k[0], _entry(pool, 100))
    assert len(st) == 2
    # a third variant under one key drops the oldest variant (max_variants=2)
    st.put(k[0], _entry(pool, 50, prefix="q"))
    st.put(k[0], _entry(pool, 50, prefix="r"))
    assert [e.prefix_hash for e in st.get(k[0])] == ["q", "r"]
    assert st.bytes == (100 + 50 + 50) * per_tok
    # LRU: k[1] is older than k[0] (get touched k[0]); going over budget evicts k[1]
    st.put(k[2], _entry(pool, 150))
    assert st.get(k[1]) == [] and st.get(k[0]) and st.get(k[2])
    assert st.bytes <= st.budget
    assert pool.released  # evicted pages went back to the pool


def test_kvstore_entry_bytes_match_reference_count():
    from chunkkv_b200.store.kvstore import Entry
    from chunkkv_b200.types import TrustLevel

    ks = [torch.zeros((1, 2, 33, 16), dtype=torch.bfloat16) for _ in range(3)]
    e = Entry(ChunkKV(ks, ks, 0), "c", "p", TrustLevel.SYSTEM)
    assert e.nbytes == sum(k.nbytes + v.nbytes for k, v in zip(ks, ks))
    pool = FakePool()
    pool.n_layers, pool.n_kv_heads, pool.head_dim = 3, 2, 16
    assert _entry(pool, 33).nbytes == e.nbytes


# ---- weights
def test_param_shapes_cover_hf_model_and_gate_up_interleave():
    from chunkkv_b200.engine.weights import hf_model, random_state_dict

    shape = SHAPES["tiny"]
    sd = random_state_dict(shape, seed=0, dtype=torch.float32)
    model = hf_model(shape, sd)
    names = {n for n, _ in param_shapes(shape)}
    assert names == set(model.state_dict()) - {"model.rotary_emb.inv_freq"}
    g = torch.arange(256 * 4, dtype=torch.float32).view(256, 4)
    u = -g
    w = interleave_gate_up(g, u)
    assert torch.equal(w[:128], g[:128]) and torch.equal(w[128:256], u[:128])
    assert torch.equal(w[256:384], g[128:]) and torch.equal(w[384:], u[128:])


def test_blend_config_defaults_are_the_reference_defaults():
    c = BlendConfig()
    assert (c.recompute_ratio, c.n_sink, c.full_first_layer, c.escalate_threshold) == (0.15, 2, True, None)
