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


def test_fused_norm_gemv_limits_are_refused_before_launch():
    """The RMSNorm-fused decode GEMVs keep the normalised rows in shared memory: more than 4
    rows, more than 5120 columns or a missing norm weight is refused on the host."""
    swiglu = "ckv_gemv_swiglu_rmsnorm"  # (h, norm_w, eps, w, out, m, inter, k, stream)
    for args, msg in [((16, 16, 1e-6, 16, 16, 5, 128, 64, None), "fused norm"),
                      ((16, 16, 1e-6, 16, 16, 1, 128, 5128, None), "fused norm"),
                      ((16, None, 1e-6, 16, 16, 1, 128, 64, None), "null norm")]:
        with pytest.raises(ValueError):
            _lib.call(swiglu, *args)
        assert msg in _lib.last_error()
    # (h, norm_w, eps, w, b, m, k, Hq, Hk, D, positions, rope, max_pos, q, K, V, n_ctx, stream)
    with pytest.raises(ValueError):
        _lib.call("ckv_gemv_qkv_rope_rmsnorm", 16, 16, 1e-6, 16, 16, 6, 64, 4, 2, 64, 16, 16, 64, 16, 16, 16,
                  40, None)
    assert "fused norm" in _lib.last_error()


def test_ops_refuse_cpu_tensors():
    x = torch.zeros((4, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.linear(x, x)
    with pytest.raises(ValueError, match="CUDA"):
        ops.rmsnorm(x, x[0], 1e-6)


def test_ops_check_shapes_before_launching():
    """The wrappers reject tensors the kernels would index out of bounds (wrong dtype,
    strides, shapes or too few elements) on the host, before any device check."""
    bf, i32, f32 = torch.bfloat16, torch.int32, torch.float32
    x, w = torch.zeros((4, 64), dtype=bf), torch.zeros((32, 64), dtype=bf)
    bad = [
        (lambda: ops.linear(x, torch.zeros((32, 48), dtype=bf)), "shape"),
        (lambda: ops.linear(x.float(), w), "bfloat16"),
        (lambda: ops.linear(x, w, out=torch.zeros((4, 16), dtype=bf)), "rows of 32"),
        (lambda: ops.linear_residual(x, w, torch.zeros((2, 32), dtype=bf)), "at least 128"),
        (lambda: ops.linear_residual(x.t(), w.t(), torch.zeros((64, 4), dtype=bf)), "contiguous"),
        (lambda: ops.linear_swiglu(x, w, torch.zeros((4, 32), dtype=bf)), "rows of 16"),
        (lambda: ops.gemv(x[0], w), r"\[m, k\]"),
        (lambda: ops.gemv_residual(x, w, torch.zeros((4, 31), dtype=bf)), "rows of 32"),
        (lambda: ops.gemv_swiglu(x, w, torch.zeros((4, 16), dtype=bf), norm_w=torch.zeros(63, dtype=bf)),
         "norm_w"),
        (lambda: ops.rmsnorm(x, torch.zeros(32, dtype=bf), 1e-6), "at least 64"),
        (lambda: ops.add_rmsnorm(x, x[:2], x[0], 1e-6, x.clone()), "delta"),
        (lambda: ops.embed(w, torch.zeros(4, dtype=torch.int64), None, x), "int32"),
        (lambda: ops.embed(w, torch.zeros(3, dtype=i32), None, x), "tokens"),
        (lambda: ops.log_softmax(x[0], out=torch.zeros(64, dtype=bf)), "float32"),
        (lambda: ops.greedy_next(x[0], torch.zeros(1, dtype=torch.int64)), "int32"),
        (lambda: ops.greedy_next(x[0], torch.zeros(1, dtype=i32), torch.zeros(0, dtype=i32)), "position"),
        (lambda: ops.greedy_next(x[0].float(), torch.zeros(1, dtype=i32)), "bfloat16"),
    ]
    # attention: q [m, Hq, D], caches [H, n_ctx, D], positions int32 [m]
    q, K = torch.zeros((3, 4, 16), dtype=bf), torch.zeros((2, 40, 16), dtype=bf)
    pos = torch.zeros(3, dtype=i32)
    bad += [
        (lambda: ops.attention(q, K, K[:, :30].contiguous(), pos, q.clone()), "length"),
        (lambda: ops.attention(q, K, K.transpose(1, 2).contiguous(), pos, q.clone()), "v_cache"),
        (lambda: ops.attention(q, K, K, pos.long(), q.clone()), "int32"),
        (lambda: ops.attention(q, K, K, pos[:2], q.clone()), "positions"),
        (lambda: ops.attention(q, K, K, pos, q[:2].clone()), "out"),
    ]
    # QKV + RoPE: w_qkv [(Hq + 2H) * D, k], rope table float32 [max_pos, D / 2, 2]
    Hq, H, D, k = 4, 2, 16, 64
    wq, bq = torch.zeros(((Hq + 2 * H) * D, k), dtype=bf), torch.zeros((Hq + 2 * H) * D, dtype=bf)
    tab, qo = torch.zeros((64, D // 2, 2), dtype=f32), torch.zeros((4, Hq * D), dtype=bf)
    Kc = torch.zeros((H, 40, D), dtype=bf)
    p4 = torch.zeros(4, dtype=i32)
    bad += [
        (lambda: ops.qkv_rope(x, wq[:100], bq, 4, 0, 100, Hq, H, D, p4, tab, q_out=qo), "w_qkv"),
        (lambda: ops.qkv_rope(x, wq, bq, 4, 0, 200, Hq, H, D, p4, tab, q_out=qo), "columns"),
        (lambda: ops.qkv_rope(x, wq, bq, 4, 0, 128, Hq, H, D, p4, tab.double(), q_out=qo), "float32"),
        (lambda: ops.qkv_rope(x, wq, bq, 4, 0, 128, Hq, H, D, p4, tab[:, :4], q_out=qo), "rope_tab"),
        (lambda: ops.qkv_rope(x, wq, bq, 4, 0, 128, Hq, H, D, p4, tab, q_out=qo, k_cache=Kc,
                              v_cache=Kc[:, :20].contiguous()), "length"),
        (lambda: ops.qkv_rope(x, wq, bq, 4, 64, 128, Hq, H, D, p4, tab,
                              k_compact=torch.zeros((4, 16), dtype=bf)), "k_compact"),
        (lambda: ops.gemv_qkv_rope(x, wq, bq, Hq, H, D, p4[:3], tab, qo, Kc, Kc), "positions"),
        (lambda: ops.gemv_qkv_rope(x, wq, bq, Hq, H, D, p4, tab, qo, Kc[:1], Kc), "k_cache"),
    ]
    # gather / store write / selection: pool [pages, layers, 2, H, 16, D], meta int32 [n, 8]
    pool = torch.zeros((4, 3, 2, H, ops.PAGE_TOKENS, D), dtype=bf)
    table, meta = torch.zeros(4, dtype=i32), torch.zeros((2, ops.META_STRIDE), dtype=i32)
    inv = torch.zeros(D // 2, dtype=f32)
    ko = torch.zeros((3, H, 40, D), dtype=bf)
    ptrs = torch.zeros(3, dtype=torch.int64)
    ws = ops.SelectWorkspace(40, 2, "cpu")
    kf, act, fl = torch.zeros((40, H * D), dtype=bf), torch.zeros(40, dtype=i32), torch.zeros(40, dtype=torch.uint8)
    smeta = torch.zeros((2, ops.SEL_META_STRIDE), dtype=i32)
    bad += [
        (lambda: ops.blend_gather_paged(pool[:, :, :1], table, meta, inv, ko, ko.clone(), 0, 3), "pool"),
        (lambda: ops.blend_gather_paged(pool, table, meta[:, :4], inv, ko, ko.clone(), 0, 3), "chunk_meta"),
        (lambda: ops.blend_gather_paged(pool, table, meta, inv, ko[:2], ko[:2].clone(), 0, 3), "k_out"),
        (lambda: ops.blend_gather_paged(pool, table, meta, inv, ko, ko[:, :, :20].clone(), 0, 3), "v_out|shape"),
        (lambda: ops.blend_gather_paged(pool, table, meta, inv, ko, ko.clone(), 1, 4), "past the pool"),
        (lambda: ops.blend_gather_paged(pool, table, meta, inv[:3], ko, ko.clone(), 0, 3), "inv_freq"),
        (lambda: ops.blend_gather_dense(ptrs.float(), ptrs, meta, inv, ko, ko.clone(), 0, 3), "addresses"),
        (lambda: ops.pages_write(pool, table[:1], 40, ptrs, ptrs, 40 * D), "page_ids"),
        (lambda: ops.pages_write(pool, table, 40, ptrs[:2], ptrs, 40 * D), "k_ptrs"),
        (lambda: ops.deviation_select(kf[:, :D], kf, Kc, Kc, act, fl, smeta, None, ws), "k_fresh"),
        (lambda: ops.deviation_select(kf, kf, Kc, Kc, act, fl[:30], smeta, None, ws), "pos_flags"),
        (lambda: ops.deviation_select(kf, kf, Kc, Kc, act, fl, smeta[:, :2], None, ws), "sel_meta"),
        (lambda: ops.deviation_select(kf, kf, Kc, Kc, act, fl, smeta, None, ops.SelectWorkspace(20, 2, "cpu")),
         "workspace"),
        (lambda: ops.select_from_scores(ws.diff.double(), ws.norm, fl, smeta, None, ws), "float32"),
        (lambda: ops.apply_selection(ws, 40, kf, kf[:20].clone(), kf, kf, kf, kf, Kc, Kc), "h_out"),
    ]
    for fn, msg in bad:
        with pytest.raises(ValueError, match=msg):
            fn()
    # the same calls with consistent arguments get as far as the device check
    good = [
        lambda: ops.blend_gather_paged(pool, table, meta, inv, ko, ko.clone(), 0, 3),
        lambda: ops.blend_gather_dense(ptrs, ptrs, meta, inv, ko, ko.clone(), 0, 3),
        lambda: ops.pages_write(pool, table, 40, ptrs, ptrs, 40 * D),
        lambda: ops.deviation_select(kf, kf, Kc, Kc, act, fl, smeta, None, ws),
        lambda: ops.deviation_scores(kf, kf, Kc, Kc, act, fl, ws),
        lambda: ops.select_from_scores(ws.diff, ws.norm, fl, smeta, None, ws),
        lambda: ops.apply_selection(ws, 40, kf, kf.clone(), kf, kf.clone(), kf, kf, Kc, Kc),
    ]
    good += [
        lambda: ops.linear(x, w, out=torch.zeros((4, 32), dtype=bf)),
        lambda: ops.linear_residual(x, w, torch.zeros((4, 32), dtype=bf)),
        lambda: ops.linear_swiglu(x, w, torch.zeros((4, 16), dtype=bf)),
        lambda: ops.gemv_swiglu(x, w, torch.zeros((4, 16), dtype=bf), norm_w=torch.zeros(64, dtype=bf)),
        lambda: ops.embed(w, torch.zeros(4, dtype=i32), None, x),
        lambda: ops.attention(q, K, K, pos, q.clone()),
        lambda: ops.qkv_rope(x, wq, bq, 4, 0, 128, Hq, H, D, p4, tab, q_out=qo, k_cache=Kc, v_cache=Kc),
        lambda: ops.gemv_qkv_rope(x, wq, bq, Hq, H, D, p4, tab, qo, Kc, Kc),
    ]
    for fn in good:
        with pytest.raises(ValueError, match="CUDA"):
            fn()


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


def test_evicted_paged_chunks_are_revoked_with_their_views():
    """An evicted entry's pages go back to the pool and may be rewritten, so its
    PagedChunkKV and every prefix view of it refuse to be read (on the host, before any
    kernel), while the kept entries stay readable."""
    from chunkkv_b200.store.kvstore import KVStore

    pool = FakePool()
    per_tok = 2 * 2 * 1 * 8 * 2
    st = KVStore(budget_bytes=2 * 100 * per_tok, pool=pool)
    k = [LookupKey.build([i], "m", None) for i in range(3)]
    for key in k:
        st.put(key, _entry(pool, 100))
    evicted = _entry(pool, 100)  # stands for an entry the caller kept from an earlier get()
    st2 = KVStore(budget_bytes=100 * per_tok, pool=pool)
    st2.put(k[0], evicted)
    view = evicted.kv.prefix(40)
    st2.put(k[1], _entry(pool, 100))  # over budget: k[0] goes, and with it `evicted`
    assert st2.get(k[0]) == [] and not evicted.kv.alive and not view.alive
    for read in (lambda: evicted.kv.materialize(), lambda: evicted.kv.keys[0], lambda: view.values[0],
                 lambda: evicted.kv.prefix(10)):
        with pytest.raises(ValueError, match="evicted"):
            read()
    assert evicted.kv.length == 100 and evicted.kv.nbytes == 100 * per_tok  # bookkeeping still works
    assert st.get(k[0]) == [] and all(e.kv.alive for key in k[1:] for e in st.get(key))


def test_kvstore_put_that_fails_leaves_no_empty_key():
    from chunkkv_b200.store.kvstore import Entry, KVStore
    from chunkkv_b200.store.pages import PAGE_TOKENS
    from chunkkv_b200.types import TrustLevel

    class TinyPool(FakePool):
        n_pages = 4

        def matches(self, L, H, D):
            return True

        def alloc(self, n):
            return None  # never room: the new key is the only one, so nothing can be evicted

    st = KVStore(pool=TinyPool())
    key = LookupKey.build([7], "m", None)
    ks = [torch.zeros((1, 1, 2 * PAGE_TOKENS, 8), dtype=torch.bfloat16) for _ in range(2)]
    with pytest.raises(MemoryError):
        st.put(key, Entry(ChunkKV(ks, ks, 0), "c", "p", TrustLevel.SYSTEM))
    assert key not in st._data and len(st) == 0 and st.bytes == 0


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
