"""Scenario runners shared by the CPU (oracle) and GPU (engine) tests."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from chunkkv_b200.engine.base import BlendConfig, Placement
from chunkkv_b200.engine.weights import SHAPES, random_state_dict
from conftest import load_golden
from scenarios import SCENARIOS, build


@dataclass
class ScenarioData:
    name: str
    meta: dict
    arrays: dict
    shape: object
    sd: dict            # bf16 state dict (HF names)
    tokens: list
    first_tokens: list
    chunk_src: list
    place: list
    config: BlendConfig


_SD_CACHE: dict = {}


def scenario(name: str) -> ScenarioData:
    meta, arrays = load_golden(name)
    sc = SCENARIOS[name]
    shape = SHAPES[sc.shape]
    key = (sc.shape, sc.seed)
    if key not in _SD_CACHE:
        _SD_CACHE.clear()
        _SD_CACHE[key] = random_state_dict(shape, seed=sc.seed, dtype=torch.bfloat16)
    b = build(sc, shape.vocab)
    assert b.tokens == meta["tokens"], "scenario builder drifted from the fixture"
    c = meta["config"]
    cfg = BlendConfig(recompute_ratio=c["recompute_ratio"], n_sink=c["n_sink"],
                      full_first_layer=c["full_first_layer"], escalate_threshold=c["escalate_threshold"])
    return ScenarioData(name, meta, arrays, shape, _SD_CACHE[key], b.tokens, b.first_tokens,
                        [tuple(x) for x in b.chunk_src], b.place, cfg)


def run_blend(eng, s: ScenarioData, chunk_len: int | None = None):
    """First prefill(s) -> chunks -> blend prefill with any engine of the reference API."""
    sc = SCENARIOS[s.name]
    L = chunk_len or sc.chunk_len
    firsts = [eng.prefill(t, None, BlendConfig()) for t in s.first_tokens]
    chunks = [firsts[fi].chunk(st, st + L) for fi, st in s.chunk_src]
    pl = [Placement(chunks[p["chunk"]], p["start"], p["ratio"], p["exact"]) for p in s.place]
    res = eng.prefill(s.tokens, pl, s.config)
    return firsts, chunks, pl, res


def kl(p_logits, q_logits) -> float:
    """KL(p || q) of the last row, as the reference tests compute it (test_torch_engine.py:30-32)."""
    p = torch.log_softmax(torch.as_tensor(np.asarray(p_logits, dtype=np.float32)).float(), -1)
    q = torch.log_softmax(torch.as_tensor(np.asarray(q_logits, dtype=np.float32)).float(), -1)
    return float((p.exp() * (p - q)).sum(-1).mean())
