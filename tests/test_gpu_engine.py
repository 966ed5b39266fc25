"""The CUDA engine end to end, against the reference (golden fixtures) and the oracle.

Parity criteria:
  - selected recompute positions bit-exact given identical fp32 scores: the
    engine's own layer-1 scores fed to the oracle's selection give exactly the
    engine's kept positions;
  - blended K/V within bf16 tolerance (max rel err <= 1e-2) of the oracle run on
    the same cached chunks;
  - first-token logit KL <= 1e-3 against the reference outputs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from chunkkv_b200 import _lib  # noqa: E402
from chunkkv_b200.engine.base import BlendConfig, ChunkKV, Placement  # noqa: E402
from chunkkv_b200.engine.torch_engine import TorchEngine  # noqa: E402
from chunkkv_b200.engine.weights import pack  # noqa: E402
from helpers import kl, run_blend, scenario  # noqa: E402
from oracle.blend_oracle import OracleEngine, select  # noqa: E402
from scenarios import SCENARIOS  # noqa: E402

ALL = list(SCENARIOS)


def rel_err(a, b) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


_ENG = {}


def engine_for(s) -> TorchEngine:
    key = (s.shape.name, SCENARIOS[s.name].seed)
    if key not in _ENG:
        _ENG.clear()
        torch.cuda.empty_cache()
        _ENG[key] = TorchEngine.from_packed(pack(s.shape, s.sd, device="cuda"))
    return _ENG[key]


@pytest.fixture(autouse=True)
def _device_error_free():
    yield
    _lib.check_device()


@pytest.mark.parametrize("name", ALL)
def test_engine_vs_reference_fixture(name):
    s = scenario(name)
    a = s.arrays
    eng = engine_for(s)
    _, _, _, res = run_blend(eng, s)
    st, ref = res.stats, s.meta["stats"]
    for k in ("tokens", "cached_tokens", "recomputed_cached_tokens", "prefill_token_equiv"):
        assert st[k] == ref[k], k
    assert [c["escalated"] for c in st["chunks"]] == [c["escalated"] for c in ref["chunks"]]
    ours = res.selected.cpu().numpy()
    overlap = len(np.intersect1d(ours, a["keep_abs"])) / len(a["keep_abs"])
    assert overlap >= 0.9, overlap
    k = kl(a["logits"][-1].astype(np.float32), res.logits[-1].float().cpu().numpy())
    assert k <= 1e-3, k


@pytest.mark.parametrize("name", ["tiny_fp32", "tiny_bf16", "tiny_escalate", "tiny_exact_overflow",
                                  "tiny7_fp32", "cfg1_0p5b"])
def test_engine_vs_oracle_same_inputs(name):
    """Same cached chunks (the engine's own first prefill) through engine and bf16 oracle."""
    s = scenario(name)
    eng = engine_for(s)
    firsts, chunks, pl, res = run_blend(eng, s)
    orc = OracleEngine(s.shape, s.sd, dtype=torch.bfloat16)
    cpu_chunks = [ChunkKV([k.cpu() for k in c.keys], [v.cpu() for v in c.values], c.start) for c in chunks]
    pl_cpu = [Placement(cpu_chunks[s.place[i]["chunk"]], p.start, p.ratio, p.exact) for i, p in enumerate(pl)]
    ores = orc.prefill(s.tokens, pl_cpu, s.config)

    # blended K/V at the positions neither engine recomputed: pure gather + re-RoPE
    # (the two selections can differ by near-tied scores; those positions hold fresh K/V)
    sel = res.selected.cpu().numpy()
    keep = np.zeros(len(s.tokens), bool)
    keep[sel] = True
    keep[ores.keep_abs.numpy()] = True
    moved = ~keep
    for li in (1, s.shape.n_layers - 1):
        assert rel_err(res.keys[li][0][:, moved], ores.keys[li][0][:, moved]) <= 1e-2
        assert rel_err(res.values[li][0][:, moved], ores.values[li][0][:, moved]) <= 1e-2

    # selection: exact given the engine's own fp32 scores
    ws = eng._ws
    N = len(s.tokens)
    cached = torch.zeros(N, dtype=torch.bool)
    sink = torch.zeros(N, dtype=torch.bool)
    for p in pl:
        cached[p.start:p.start + p.chunk.length] = True
        if not p.exact:
            sink[p.start:min(p.start + p.chunk.length, p.start + s.config.n_sink)] = True
    ours = select(ws.diff[:N].cpu(), ws.norm[:N].cpu(), cached, sink, pl, s.config)
    np.testing.assert_array_equal(ours["keep_abs"].numpy(), sel)
    # scores within tolerance of the oracle's on the same inputs
    act = ~np.asarray([False] * N)
    for p in pl:
        if p.exact:
            act[p.start:p.start + p.chunk.length] = False
    d_o, d_e = ores.diff.numpy()[act], ws.diff[:N].cpu().numpy()[act]
    assert np.abs(d_e - d_o).max() <= 0.05 * np.abs(d_o).max() + 1e-6
    jac = len(np.intersect1d(sel, ores.keep_abs.numpy())) / len(np.union1d(sel, ores.keep_abs.numpy()))
    assert jac >= 0.9, jac
    k = kl(ores.logits[-1].float().numpy(), res.logits[-1].float().cpu().numpy())
    assert k <= 1e-3, k


def test_no_cache_prefill_matches_oracle_all_logits():
    """test_torch_engine.py:36-41 shape: every position's logits (logits_from=0)."""
    s = scenario("tiny_fp32")
    eng = engine_for(s)
    toks = s.tokens[:100]
    out = eng.prefill(toks, logits_from=0)
    orc = OracleEngine(s.shape, s.sd, dtype=torch.float32)
    ref = orc.prefill(toks, None, BlendConfig(), logits_from=0)
    assert out.logits.shape == ref.logits.shape
    for r in (0, 50, 99):
        assert kl(ref.logits[r].numpy(), out.logits[r].float().cpu().numpy()) <= 1e-3


def test_same_position_exact_reuse():
    """test_torch_engine.py:44-49: an exact chunk at its own offset reproduces the first prefill."""
    s = scenario("tiny_fp32")
    eng = engine_for(s)
    toks = s.tokens
    first = eng.prefill(toks)
    st = 16
    out = eng.prefill(toks, [Placement(first.chunk(st, st + 48), st, exact=True)], BlendConfig())
    assert kl(first.logits[-1].float().cpu().numpy(), out.logits[-1].float().cpu().numpy()) <= 1e-4
    assert out.stats["prefill_token_equiv"] == (len(toks) - 48 + (len(toks) - 48) * 3) / 4


def test_moved_chunk_blend_beats_naive():
    """test_torch_engine.py:52-65 on random weights: ratio 1.0 ~ full, blend closer than naive."""
    s = scenario("tiny_fp32")
    eng = engine_for(s)
    firsts = [eng.prefill(t) for t in s.first_tokens]
    chunks = [firsts[fi].chunk(st, st + 48) for fi, st in s.chunk_src]
    pl = [Placement(chunks[p["chunk"]], p["start"]) for p in s.place]
    p0 = eng.prefill(s.tokens).logits[-1].float().cpu().numpy()
    full = eng.prefill(s.tokens, pl, BlendConfig(recompute_ratio=1.0)).logits[-1].float().cpu().numpy()
    naive = eng.prefill(s.tokens, pl, BlendConfig(full_first_layer=False))
    blend = eng.prefill(s.tokens, pl, BlendConfig(recompute_ratio=0.3))
    assert kl(p0, full) < 1e-3
    assert kl(p0, blend.logits[-1].float().cpu().numpy()) < kl(p0, naive.logits[-1].float().cpu().numpy())
    assert naive.stats["prefill_token_equiv"] < blend.stats["prefill_token_equiv"] < len(s.tokens)


def test_paged_store_placements_equal_dense():
    """Chunks served from the paged HBM store give the same result as dense per-layer chunks."""
    from chunkkv_b200.store.keys import LookupKey
    from chunkkv_b200.store.kvstore import Entry, KVStore
    from chunkkv_b200.types import TrustLevel

    s = scenario("tiny7_fp32")
    eng = engine_for(s)
    firsts, chunks, pl, dense = run_blend(eng, s)
    store = KVStore(budget_bytes=64 << 20)
    paged = []
    for i, c in enumerate(chunks):
        key = LookupKey.build(list(range(i, i + 5)), "m", None)
        store.put(key, Entry(c, "ctx", f"p{i}", TrustLevel.SYSTEM))
        paged.append(store.get(key)[0].kv)
    for i, c in enumerate(chunks):
        for li in range(s.shape.n_layers):
            assert torch.equal(paged[i].keys[li], c.keys[li])
    pl2 = [Placement(paged[s.place[i]["chunk"]], p.start, p.ratio, p.exact) for i, p in enumerate(pl)]
    out = eng.prefill(s.tokens, pl2, s.config)
    assert torch.equal(out.logits, dense.logits)
    assert torch.equal(out.cache[0], dense.cache[0]) and torch.equal(out.cache[1], dense.cache[1])


def test_result_chunks_are_views_until_read_then_copies():
    """PrefillResult.chunk: the store writes pages from the cache view; reading keys
    gives (1, H, len, D) copies that no longer depend on the request's cache."""
    from chunkkv_b200.engine.base import CacheChunkKV
    from chunkkv_b200.store.keys import LookupKey
    from chunkkv_b200.store.kvstore import Entry, KVStore
    from chunkkv_b200.types import TrustLevel

    s = scenario("tiny_bf16")
    eng = engine_for(s)
    res = eng.prefill(s.first_tokens[0])
    K, V = res.cache
    stored = res.chunk(5, 70)
    assert isinstance(stored, CacheChunkKV) and stored.length == 65 and stored.start == 5
    store = KVStore(budget_bytes=64 << 20)
    key = LookupKey.build([1, 2, 3], "m", None)
    store.put(key, Entry(stored, "ctx", "p", TrustLevel.SYSTEM))
    paged = store.get(key)[0].kv
    kept = res.chunk(5, 70)
    ks, vs = kept.keys, kept.values
    assert not kept.viewable and len(ks) == s.shape.n_layers
    for li in range(s.shape.n_layers):
        assert ks[li].shape == (1, s.shape.n_kv, 65, s.shape.head_dim) and ks[li].is_contiguous()
        assert torch.equal(ks[li][0], K[li, :, 5:70]) and torch.equal(vs[li][0], V[li, :, 5:70])
        assert torch.equal(paged.keys[li], ks[li]) and torch.equal(paged.values[li], vs[li])
    with torch.inference_mode():
        K.zero_()
    assert ks[0].abs().sum() > 0  # the copy is detached from the cache


def test_evicted_store_chunk_is_refused_by_prefill():
    """An entry evicted from the store gives its pages back; a caller still holding its
    PagedChunkKV cannot place it in a prefill (ValueError before any launch), while the
    entry that replaced it serves as usual."""
    from chunkkv_b200.store.keys import LookupKey
    from chunkkv_b200.store.kvstore import Entry, KVStore
    from chunkkv_b200.types import TrustLevel

    s = scenario("tiny_bf16")
    eng = engine_for(s)
    doc = s.first_tokens[0][:64]
    res = eng.prefill(doc)
    per_entry = s.shape.n_layers * 2 * s.shape.n_kv * 64 * s.shape.head_dim * 2
    store = KVStore(budget_bytes=per_entry)  # room for exactly one entry
    k1, k2 = LookupKey.build([1], "m", None), LookupKey.build([2], "m", None)
    store.put(k1, Entry(res.chunk(0, 64), "c", "p1", TrustLevel.SYSTEM))
    old = store.get(k1)[0].kv
    store.put(k2, Entry(res.chunk(0, 64), "c", "p2", TrustLevel.SYSTEM))
    assert store.get(k1) == [] and not old.alive
    query = doc + [1, 2, 3]
    with pytest.raises(ValueError, match="evicted"):
        eng.prefill(query, [Placement(old, 0)], BlendConfig())
    new = store.get(k2)[0].kv
    out = eng.prefill(query, [Placement(new, 0)], BlendConfig())
    assert torch.isfinite(out.logits.float()).all()


def test_logits_for_unrecomputed_positions_raise():
    s = scenario("tiny_fp32")
    eng = engine_for(s)
    _, _, pl, _ = run_blend(eng, s)
    with pytest.raises(ValueError):
        eng.prefill(s.tokens, pl, s.config, logits_from=s.place[0]["start"] + 10)


def test_generate_matches_oracle_greedy():
    s = scenario("tiny_fp32")
    eng = engine_for(s)
    toks = s.tokens[:60]
    ours = eng.generate(eng.prefill(toks), max_tokens=8)
    orc = OracleEngine(s.shape, {k: v.float() for k, v in s.sd.items()}, dtype=torch.float32)
    seq = list(toks)
    ref = []
    for _ in range(8):
        nxt = int(orc.prefill(seq, None, BlendConfig()).logits[-1].argmax())
        ref.append(nxt)
        seq.append(nxt)
    agree = 0
    for x, y in zip(ours, ref):
        if x != y:
            break
        agree += 1
    assert len(ours) == 8 and agree >= 4, (ours, ref)


def test_hf_model_constructor_and_last_logprobs():
    from chunkkv_b200.engine.weights import hf_model

    s = scenario("tiny_fp32")
    eng = TorchEngine(hf_model(s.shape, s.sd, dtype=torch.bfloat16).cuda())
    res = eng.prefill(s.tokens[:40])
    lp = eng.last_logprobs(res)
    assert lp.shape == (s.shape.vocab,) and abs(np.exp(lp).sum() - 1) < 1e-3
    assert eng.n_kv == s.shape.n_kv and eng.head_dim == s.shape.head_dim
    k = torch.randn((1, eng.n_kv, 10, eng.head_dim), device="cuda").to(torch.bfloat16)
    assert eng.shift_keys(k, 0) is k
