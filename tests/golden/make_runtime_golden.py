"""Generate runtime_policies.json by running the REFERENCE runtimes (P0-P4).

    python tests/golden/make_runtime_golden.py --ref /path/to/chunkkv

Needs the reference source tree (sarvanithin/chunkkv: src/ and bench/); it runs
only where that exists, never in the tests.  The request stream of
runtime_stream.py goes through bench/policies.py:build(policy, ...) of the
reference with a stand-in engine that records every prefill call (tokens,
placements, blend settings) and returns zero K/V of 2 layers x 1 head x 8 dims,
so the fixture pins the runtime, gate and store bookkeeping
(runtime.py:50-132, gate.py:38-72, kvstore.py:20-63) independently of the model.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

from runtime_stream import CHUNK_BUDGET, PREFIX_BUDGET, build_request, stream  # noqa: E402


def describe(placements, blend) -> dict:
    return {
        "placements": [[p.start, p.ratio, bool(p.exact), p.chunk.start, p.chunk.keys[0].shape[2]]
                       for p in placements],
        "blend": [blend.recompute_ratio, blend.full_first_layer, blend.escalate_threshold],
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="the reference project checkout (sarvanithin/chunkkv)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.ref) / "src"))
    sys.path.insert(0, args.ref)
    from bench.policies import POLICIES, build
    from chunkkv import types
    from chunkkv.engine.base import PrefillResult

    class Engine:
        def __init__(self):
            self.calls = []

        def prefill(self, tokens, placements=None, config=None, logits_from=None):
            self.calls.append({"n": len(tokens), "logits_from": logits_from, **describe(placements or [], config)})
            k = [torch.zeros((1, 1, len(tokens), 8), dtype=torch.bfloat16) for _ in range(2)]
            return PrefillResult(None, None, k, [t.clone() for t in k], {}, copy=lambda a: a.clone())

    out = {"stream_seed": 0, "policies": {}}
    reqs = stream(0)
    for pol in POLICIES:
        eng = Engine()
        budget = PREFIX_BUDGET if pol == "P1" else CHUNK_BUDGET
        rt = build(pol, eng, "m", budget_bytes=budget, ratio=0.15)
        decisions = []
        for r in reqs:
            o = rt.prefill(build_request(r, types))
            decisions.append([[d.segment, d.action.value, d.reason, d.ratio] for d in o.decisions])
        rec = {"calls": eng.calls, "decisions": decisions}
        if pol == "P1":
            rec["kept"] = [len(seq) for seq, _ in rt._seqs.values()]
            rec["bytes"] = rt.bytes
        else:
            rec["store"] = [[[e.context_id, e.prefix_hash, int(e.context_trust), e.hits, e.kv.start,
                              e.kv.keys[0].shape[2]] for e in entries]
                            for entries in rt.store._data.values()]
            rec["bytes"] = rt.store.bytes
        out["policies"][pol] = rec
    (HERE / "runtime_policies.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", HERE / "runtime_policies.json")


if __name__ == "__main__":
    main()
