"""Generate report_summary.json with the REFERENCE's bench/report.py.

    python tests/golden/make_report_golden.py --ref /path/to/chunkkv

Seeded synthetic replay rows (the fields bench/replay.py writes) go through the
reference's summarize() and boot_ci(); rows and results are saved so the tests can
check chunkkv_b200.harness against them.  Needs the reference tree; never run by
the tests.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def rows(policy: str, seed: int, n: int = 23) -> list[dict]:
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        r = {"id": f"r{i}", "policy": policy, "tokens": int(rng.integers(200, 4000)),
             "ttft": float(rng.gamma(2.0, 0.01)), "compute": float(rng.uniform(0.05, 1.0)),
             "decisions": [[str(rng.choice(["reuse", "blend", "recompute"])),
                            str(rng.choice(["exact_prefix", "same_context", "other_context", "trust"]))]
                           for _ in range(int(rng.integers(0, 4)))],
             "conflict": bool(rng.random() < 0.3), "correct": bool(rng.random() < 0.7)}
        if policy != "P0":
            r.update(kl=float(rng.exponential(0.01)), match_p0=bool(rng.random() < 0.6),
                     agree_prefix=float(rng.uniform()))
        if rng.random() < 0.4:
            r["attacked"] = bool(rng.random() < 0.2)
        out.append(r)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="the reference project checkout (sarvanithin/chunkkv)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.ref) / "src"))
    sys.path.insert(0, args.ref)
    from bench.report import boot_ci, summarize

    cases = []
    for pol, seed, skip in (("P0", 1, 0), ("P3", 2, 0), ("P4", 3, 2)):
        rs = rows(pol, seed)
        cases.append({"rows": rs, "skip_first": skip, "summary": summarize(rs, skip)})
    x = np.random.default_rng(9).random(37) < 0.55
    out = {"cases": cases, "boot": {"x": x.tolist(), "ci": boot_ci(x.astype(float))}}
    (HERE / "report_summary.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", HERE / "report_summary.json")


if __name__ == "__main__":
    main()
