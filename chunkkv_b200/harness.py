"""Policy replay and report (the reference's bench/replay.py:28-71 and
bench/report.py:17-57, over synthetic request streams).

`replay_policy` serves a list of ChunkedRequests under one policy runtime and
returns one row per request with the reference's fields: time to first token
(prefill + first-token log-probs, wall clock, as replay.py:33-35), compute share
(`prefill_token_equiv / tokens`), cached and recomputed-cached tokens, the gate
decisions, and against the P0 run of the same request the first-token KL, whether
the greedy continuation is identical, and the share of it that agrees before the
first difference.  Outputs are compared as token lists (the synthetic streams have
no text).  `summarize` and `boot_ci` aggregate rows as report.py does (percentile
bootstrap, 2000 resamples, seed 0).
"""

from __future__ import annotations

import time
from collections import Counter

import numpy as np


def boot_ci(x: np.ndarray, stat=np.mean, n: int = 2000, seed: int = 0) -> tuple[float, float]:
    """95 % percentile-bootstrap interval of `stat` (report.py:17-22)."""
    x = np.asarray(x)
    if len(x) == 0:
        return float("nan"), float("nan")
    rng = np.random.default_rng(seed)
    s = [stat(x[rng.integers(0, len(x), len(x))]) for _ in range(n)]
    return float(np.percentile(s, 2.5)), float(np.percentile(s, 97.5))


def summarize(rows: list[dict], skip_first: int = 0) -> dict:
    """One policy's rows -> n, TTFT p50/p95, token-weighted compute share, KL and
    P0 agreement with its interval, accuracy / attack rates when present, and the
    decision counts (report.py:29-57)."""
    rows = rows[skip_first:]
    ttft = np.array([r["ttft"] for r in rows])
    toks = np.array([r["tokens"] for r in rows], dtype=np.float64)
    s = {
        "n": len(rows),
        "ttft_p50": float(np.median(ttft)), "ttft_p95": float(np.percentile(ttft, 95)),
        "compute": float(np.sum(np.array([r["compute"] for r in rows]) * toks) / np.sum(toks)),
    }
    if "kl" in rows[0]:
        s["kl"] = float(np.mean([r["kl"] for r in rows]))
        m = np.array([r["match_p0"] for r in rows], float)
        s["match_p0"], s["match_ci"] = float(m.mean()), boot_ci(m)
        conf = np.array([r["match_p0"] for r in rows if r.get("conflict")], float)
        if len(conf):
            s["match_p0_conflict"] = float(conf.mean())
    if "correct" in rows[0]:
        c = np.array([r["correct"] for r in rows], float)
        s["acc"], s["acc_ci"] = float(c.mean()), boot_ci(c)
    att = [r["attacked"] for r in rows if "attacked" in r]
    if att:
        s["attack_success"] = float(np.mean(att))
    s["decisions"] = dict(Counter(a for r in rows for a, _ in r["decisions"]))
    s["reasons"] = dict(Counter(why for r in rows for _, why in r["decisions"]))
    return s


def compare_to_p0(logp: np.ndarray, gen: list[int], p0_logp: np.ndarray, p0_gen: list[int]) -> dict:
    """KL(P0 || policy) of the first-token distribution, exact output match, and the
    agreeing share of P0's output before the first difference (replay.py:55-63)."""
    n = 0
    for a, b in zip(gen, p0_gen):
        if a != b:
            break
        n += 1
    return {"kl": float(np.sum(np.exp(p0_logp) * (p0_logp - logp))), "match_p0": gen == p0_gen,
            "agree_prefix": n / max(1, len(p0_gen))}


def replay_policy(policy: str, runtime, engine, requests: list, ref: dict, max_new: int = 8,
                  sync=None) -> list[dict]:
    """Serve `requests` (list of (id, ChunkedRequest)) in order under `runtime`.  P0
    fills `ref[id] = (logp, gen)`; other policies are compared with it."""
    rows = []
    for rid, req in requests:
        if sync is not None:
            sync()
        t0 = time.perf_counter()
        out = runtime.prefill(req)
        logp = engine.last_logprobs(out.result)  # waits for the prefill
        ttft = time.perf_counter() - t0
        gen = engine.generate(out.result, max_new) if max_new > 0 else []
        st = out.stats
        row = {
            "id": rid, "policy": policy, "tokens": len(req.tokens), "ttft": ttft,
            "compute": st["prefill_token_equiv"] / len(req.tokens),
            "cached_tokens": st["cached_tokens"], "recomputed_cached": st["recomputed_cached_tokens"],
            "decisions": [[d.action.value, d.reason] for d in out.decisions], "chunks": st["chunks"],
        }
        if policy == "P0":
            ref[rid] = (logp, gen)
        else:
            row.update(compare_to_p0(logp, gen, *ref[rid]))
        rows.append(row)
        del out
    return rows
