"""Generate the golden fixtures by running the REFERENCE TorchEngine on CPU.

    python tests/golden/make_golden.py --ref /path/to/chunkkv/src [names...]

Needs the reference source tree (sarvanithin/chunkkv, src/ importable) and the
transformers Qwen2 model; it runs only where those exist, never in the tests.
For each scenario of scenarios.py it builds a Hugging Face Qwen2ForCausalLM with
chunkkv_b200.engine.weights.random_state_dict(shape, seed) (bf16 values), runs
the first prefill(s) and the blend prefill through chunkkv.engine.torch_engine.
TorchEngine, and records its outputs.  The layer-1 deviation vectors are read
from the two fp32 `torch.zeros(N)` buffers TorchEngine.prefill allocates at
torch_engine.py:121-122, the top-k order from its `torch.argsort` call
(torch_engine.py:144); both are observed with wrappers, the reference code is
not changed.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from unittest import mock

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE))

from chunkkv_b200.engine.weights import SHAPES, hf_model, random_state_dict  # noqa: E402
from scenarios import SCENARIOS, build  # noqa: E402


class _Tok:
    eos_token_id = 0


def run(name: str, ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    from chunkkv.engine.base import BlendConfig, Placement  # reference types
    from chunkkv.engine.torch_engine import TorchEngine

    sc = SCENARIOS[name]
    shape = SHAPES[sc.shape]
    torch.manual_seed(0)
    sd = random_state_dict(shape, seed=sc.seed, dtype=torch.bfloat16)
    dtype = torch.float32 if sc.dtype == "fp32" else torch.bfloat16
    model = hf_model(shape, sd, dtype=dtype)
    eng = TorchEngine(model, _Tok())
    b = build(sc, shape.vocab)

    firsts = [eng.prefill(t) for t in b.first_tokens]
    chunks = [firsts[fi].chunk(s, s + sc.chunk_len) for fi, s in b.chunk_src]
    placements = [Placement(chunks[p["chunk"]], p["start"], p["ratio"], p["exact"]) for p in b.place]
    cfg = BlendConfig(recompute_ratio=sc.ratio, n_sink=sc.n_sink, full_first_layer=sc.full_first_layer,
                      escalate_threshold=sc.escalate)

    made, orders = [], []
    real_zeros, real_argsort = torch.zeros, torch.argsort

    def zeros_spy(*a, **k):
        t = real_zeros(*a, **k)
        if t.dim() == 1 and t.dtype == torch.float32:
            made.append(t)
        return t

    def argsort_spy(x, *a, **k):
        out = real_argsort(x, *a, **k)
        orders.append((x.detach().clone(), out.detach().clone()))
        return out

    with mock.patch.object(torch, "zeros", zeros_spy), mock.patch.object(torch, "argsort", argsort_spy):
        res = eng.prefill(b.tokens, placements, cfg)
    p0 = eng.prefill(b.tokens)  # full recompute (P0) of the same request

    N = len(b.tokens)
    diff, norm = (made[0], made[1]) if len(made) >= 2 else (real_zeros(N), real_zeros(N))
    budget = 0
    top = np.zeros(0, dtype=np.int64)
    scores = np.zeros(0, dtype=np.float32)
    if orders:
        neg, order = orders[0]
        scores = (-neg).float().numpy()
        elig = scores >= 0
        # budget after the cap, as torch_engine.py:139-142 computes it
        budget = 0
        for p in placements:
            if p.exact:
                continue
            r = cfg.recompute_ratio if p.ratio is None else p.ratio
            st = next(c for c in res.stats["chunks"] if c["start"] == p.start)
            if not st["escalated"] and r > 0:
                budget += int(round(r * p.chunk.length))
        budget = min(budget, int(elig.sum()))
        top = order[:budget].numpy()
    # keep = ~cached | sink | escalated | top  (torch_engine.py:125-146)
    cached = np.zeros(N, bool)
    sink = np.zeros(N, bool)
    keep = np.zeros(N, bool)
    for p in placements:
        cached[p.start:p.start + p.chunk.length] = True
        if not p.exact:
            sink[p.start:min(p.start + p.chunk.length, p.start + cfg.n_sink)] = True
    keep |= ~cached | sink
    for c in res.stats["chunks"]:
        if c["escalated"]:
            keep[c["start"]:c["start"] + c["length"]] = True
    keep[top] = True
    if not cfg.full_first_layer or not placements:
        keep[:] = ~cached

    logits = res.logits.float()
    p0_logits = p0.logits.float()
    small = np.float32 if sc.store_full_logits else np.float16
    span = slice(0, N) if sc.store_full_logits else slice(b.place[0]["start"], b.place[0]["start"] + sc.chunk_len)
    arrays = dict(
        diff=diff.float().numpy(), norm=norm.float().numpy(), scores=scores, top=top,
        keep_abs=np.flatnonzero(keep).astype(np.int32),
        logits=(logits.numpy() if sc.store_full_logits else logits.half().numpy()),
        p0_logits=(p0_logits.numpy() if sc.store_full_logits else p0_logits.half().numpy()),
        first_logits=firsts[0].logits.float()[-1].numpy().astype(np.float32 if sc.store_full_logits
                                                                   else np.float16),
        # per-layer sum of squares of the first prefill's K and V (pins the chunk K/V inputs)
        first_k_ss=np.array([float((k.float() ** 2).sum()) for k in firsts[0].keys]),
        first_v_ss=np.array([float((v.float() ** 2).sum()) for v in firsts[0].values]),
        # blended layer-1 cache (pins the gather / re-RoPE); for the large scenario only the
        # span of the first placement, to keep the fixture small
        blend_k1=res.keys[1][0, :, span].float().numpy().astype(small),
        blend_v1=res.values[1][0, :, span].float().numpy().astype(small),
        blend_span=np.array([span.start, span.stop]),
    )
    meta = dict(
        scenario=name, reference="sarvanithin/chunkkv src/chunkkv/engine/torch_engine.py",
        torch=torch.__version__, stats=res.stats, p0_stats=p0.stats, budget=int(budget),
        tokens=b.tokens, first_tokens=b.first_tokens, chunk_src=b.chunk_src, place=b.place,
        config=dict(recompute_ratio=cfg.recompute_ratio, n_sink=cfg.n_sink,
                    full_first_layer=cfg.full_first_layer, escalate_threshold=cfg.escalate_threshold),
    )
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    (HERE / f"{name}.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print(f"{name}: N={N} budget={budget} selected={int(keep.sum())} "
          f"stats={ {k: v for k, v in res.stats.items() if k != 'chunks'} }")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="the reference project's src/ directory")
    ap.add_argument("names", nargs="*", default=list(SCENARIOS))
    a = ap.parse_args()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    for n in a.names:
        run(n, a.ref)


if __name__ == "__main__":
    main()
