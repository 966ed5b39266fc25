"""The runtimes (policies P0-P4) on the CUDA engine and the paged store.

  - P1 (prefix cache): a request that extends an earlier one is served its longest
    common prefix from the pages and gives the same first-token distribution as a
    full prefill (KL <= 1e-4, the exact-reuse bound of test_gpu_engine.py);
  - P3 at recompute ratio 1.0: every request of the seeded multi-tenant stream
    matches P0 (KL <= 1e-3, the full-ratio bound of test_torch_engine.py:52-65);
  - for every policy, the engine's `cached_tokens` is the length of what the
    runtime placed, and the store never exceeds its budget.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))

from chunkkv_b200 import _lib, types  # noqa: E402
from chunkkv_b200.engine.torch_engine import TorchEngine  # noqa: E402
from chunkkv_b200.engine.weights import SHAPES, pack, random_state_dict  # noqa: E402
from chunkkv_b200.policies import build  # noqa: E402
from helpers import kl  # noqa: E402
from runtime_stream import build_request, stream  # noqa: E402

_ENG: list = []


def engine() -> TorchEngine:
    if not _ENG:
        shape = SHAPES["tiny"]
        _ENG.append(TorchEngine.from_packed(pack(shape, random_state_dict(shape, seed=3, dtype=torch.bfloat16),
                                                 device="cuda")))
    return _ENG[0]


class Recording:
    """Engine wrapper that keeps the placements of the last prefill."""

    def __init__(self, eng):
        self._e, self.device, self.placed = eng, eng.device, 0

    def prefill(self, tokens, placements=None, config=None, logits_from=None):
        self.placed = sum(p.chunk.length for p in placements or [])
        return self._e.prefill(tokens, placements, config, logits_from)


def _requests(vocab: int):
    out = []
    for r in stream(0):
        r = dict(r, segments=[(role, tr, [t % vocab for t in toks], ru) for role, tr, toks, ru in r["segments"]])
        out.append(build_request(r, types))
    return out


@pytest.fixture(autouse=True)
def _device_error_free():
    yield
    _lib.check_device()


def test_prefix_cache_serves_the_longest_prefix_from_pages():
    eng = engine()
    rng = np.random.default_rng(1)
    base = rng.integers(1, 1000, 160).tolist()
    rt = build("P1", eng, "tiny", budget_bytes=64 << 20)

    def req(toks):
        return types.ChunkedRequest(toks, [types.Segment(0, "user", types.TrustLevel.USER, 0, toks, False)],
                                    "t", "c")

    rt.prefill(req(base[:100]))
    longer = base[:100] + rng.integers(1, 1000, 40).tolist()
    out = rt.prefill(req(longer))
    assert out.stats["cached_tokens"] == 100
    full = eng.prefill(longer)
    assert kl(full.logits[-1].float().cpu().numpy(), out.result.logits[-1].float().cpu().numpy()) <= 1e-4
    # a third request shares 60 tokens with both: the first kept sequence serves it
    third = base[:60] + rng.integers(1, 1000, 30).tolist()
    out3 = rt.prefill(req(third))
    assert out3.stats["cached_tokens"] == 60
    assert kl(eng.prefill(third).logits[-1].float().cpu().numpy(),
              out3.result.logits[-1].float().cpu().numpy()) <= 1e-4


def test_full_ratio_blend_policy_matches_no_cache_on_the_stream():
    eng = engine()
    reqs = _requests(SHAPES["tiny"].vocab)
    p0 = build("P0", eng, "tiny")
    ref = [eng.last_logprobs(p0.prefill(r).result) for r in reqs]
    rec = Recording(eng)
    p3 = build("P3", rec, "tiny", budget_bytes=64 << 20, ratio=1.0)
    served = 0
    for r, lp0 in zip(reqs, ref):
        out = p3.prefill(r)
        assert out.stats["cached_tokens"] == rec.placed
        served += rec.placed
        lp = eng.last_logprobs(out.result)
        assert float(np.sum(np.exp(lp0) * (lp0 - lp))) <= 1e-3
    assert served > 0  # the stream does reuse chunks


@pytest.mark.parametrize("policy", ["P1", "P2", "P4"])
def test_policies_place_what_the_engine_counts(policy):
    eng = engine()
    rec = Recording(eng)
    budget = 2 << 20  # small: the stores evict during the stream
    rt = build(policy, rec, "tiny", budget_bytes=budget, ratio=0.15)
    for r in _requests(SHAPES["tiny"].vocab):
        out = rt.prefill(r)
        assert out.stats["cached_tokens"] == rec.placed
        assert np.isfinite(eng.last_logprobs(out.result)).all()
        assert (rt.bytes if policy == "P1" else rt.store.bytes) <= budget
