"""The CPU oracle against the reference's own outputs (golden fixtures).

The fixtures were produced by running sarvanithin/chunkkv's TorchEngine on CPU
(tests/golden/make_golden.py); these tests re-run the same scenarios through
oracle/blend_oracle.py and require the same results.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import kl, run_blend, scenario
from oracle.blend_oracle import OracleEngine, plan_positions, select
from scenarios import SCENARIOS

FP32_CASES = [n for n, s in SCENARIOS.items() if s.dtype == "fp32"]


def _oracle(s):
    dtype = torch.float32 if SCENARIOS[s.name].dtype == "fp32" else torch.bfloat16
    return OracleEngine(s.shape, {k: v.to(dtype) for k, v in s.sd.items()}, dtype=dtype)


@pytest.mark.parametrize("name", list(SCENARIOS))
def test_oracle_matches_reference(name):
    s = scenario(name)
    a = s.arrays
    eng = _oracle(s)
    firsts, _, _, res = run_blend(eng, s)
    bf16 = SCENARIOS[name].dtype == "bf16"
    big = not SCENARIOS[name].store_full_logits

    # inputs: the first prefill (which produces the cached chunks)
    first = firsts[0].logits.float()[-1].numpy()
    # fp16-stored fixtures (the large scenario) carry ~5e-4 relative quantisation
    np.testing.assert_allclose(first, a["first_logits"].astype(np.float32),
                               atol=0.02 if big else (2e-2 if bf16 else 1e-4), rtol=2e-3 if big else 0)
    ss = np.array([float((k.float() ** 2).sum()) for k in firsts[0].keys])
    np.testing.assert_allclose(ss, a["first_k_ss"], rtol=1e-3 if bf16 else 1e-5)

    # selection: exact indices, same budget, same integer stats
    st, ref_st = res.stats, s.meta["stats"]
    for k in ("tokens", "cached_tokens", "recomputed_cached_tokens", "prefill_token_equiv"):
        assert st[k] == ref_st[k], k
    assert res.budget == s.meta["budget"]
    np.testing.assert_array_equal(res.keep_abs.numpy(), a["keep_abs"])
    assert [c["escalated"] for c in st["chunks"]] == [c["escalated"] for c in ref_st["chunks"]]
    np.testing.assert_allclose([c["rel_dev"] for c in st["chunks"]],
                               [c["rel_dev"] for c in ref_st["chunks"]], rtol=1e-2 if bf16 else 1e-4)

    # layer-1 deviation scores and the blended layer-1 cache
    np.testing.assert_allclose(res.diff.numpy(), a["diff"], rtol=2e-2 if bf16 else 1e-3, atol=1e-6)
    np.testing.assert_allclose(res.norm.numpy(), a["norm"], rtol=1e-2 if bf16 else 1e-4)
    lo, hi = a["blend_span"]
    np.testing.assert_allclose(res.keys[1][0, :, lo:hi].float().numpy(), a["blend_k1"].astype(np.float32),
                               atol=2e-2 if (bf16 or big) else 1e-4, rtol=1e-2 if (bf16 or big) else 1e-4)

    # output: first-token distribution
    assert kl(a["logits"][-1], res.logits[-1].float().numpy()) < (1e-4 if not bf16 else 1e-3)


@pytest.mark.parametrize("name", FP32_CASES)
def test_oracle_selection_from_reference_scores(name):
    """Given the reference's own fp32 scores, the oracle selects the reference's tokens."""
    s = scenario(name)
    a = s.arrays
    N = len(s.tokens)

    class P:  # minimal placement view for the selection restatement
        def __init__(self, p):
            self.start, self.ratio, self.exact = p["start"], p["ratio"], p["exact"]
            self.chunk = type("C", (), {"length": SCENARIOS[name].chunk_len})()

    pl = [P(p) for p in s.place]
    cached_l, _, sink_l = plan_positions(N, pl, s.config.n_sink)
    out = select(torch.from_numpy(a["diff"]), torch.from_numpy(a["norm"]), torch.tensor(cached_l),
                 torch.tensor(sink_l), pl, s.config)
    np.testing.assert_array_equal(out["keep_abs"].numpy(), a["keep_abs"])
    assert out["budget"] == s.meta["budget"]
    if len(a["top"]):
        assert set(a["top"].tolist()) == set(np.flatnonzero(out["eligible"].numpy() &
                                                            np.isin(np.arange(N), out["keep_abs"].numpy())).tolist())


def test_full_blend_is_close_to_full_prefill():
    """Property of test_torch_engine.py:52-65: ratio 1.0 blend ~ full recompute (KL < 1e-4),
    and a partial blend is closer to it than naive reuse."""
    s = scenario("tiny_fp32")
    eng = _oracle(s)
    from chunkkv_b200.engine.base import BlendConfig, Placement

    firsts = [eng.prefill(t, None, BlendConfig()) for t in s.first_tokens]
    L = SCENARIOS["tiny_fp32"].chunk_len
    chunks = [firsts[fi].chunk(st, st + L) for fi, st in s.chunk_src]
    pl = [Placement(chunks[p["chunk"]], p["start"]) for p in s.place]
    p0 = eng.prefill(s.tokens, None, BlendConfig()).logits[-1]
    full = eng.prefill(s.tokens, pl, BlendConfig(recompute_ratio=1.0)).logits[-1]
    naive = eng.prefill(s.tokens, pl, BlendConfig(full_first_layer=False)).logits[-1]
    blend = eng.prefill(s.tokens, pl, BlendConfig(recompute_ratio=0.3)).logits[-1]
    assert kl(p0, full) < 1e-4
    assert kl(p0, blend) < kl(p0, naive)


def test_oracle_matches_hf_forward():
    """No-cache prefill == the Hugging Face forward (test_torch_engine.py:36-41)."""
    from chunkkv_b200.engine.base import BlendConfig
    from chunkkv_b200.engine.weights import hf_model

    s = scenario("tiny_fp32")
    eng = _oracle(s)
    model = hf_model(s.shape, s.sd, dtype=torch.float32)
    toks = s.tokens[:64]
    with torch.inference_mode():
        ref = model(torch.tensor([toks])).logits[0]
    out = eng.prefill(toks, None, BlendConfig(), logits_from=0)
    torch.testing.assert_close(out.logits, ref, atol=2e-3, rtol=0)
