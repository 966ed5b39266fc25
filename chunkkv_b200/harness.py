"""Policy replay and report (the reference's bench/replay.py:28-71 and
bench/report.py:17-57, over synthetic request streams).

`replay_policy` serves a list of ChunkedRequests under one policy runtime and
returns one row per request with the reference's fields: time to first token
(prefill + first-token log-probs, wall clock, as replay.py:33-35), compute share
(`prefill_token_equiv / tokens`), cached and recomputed-cached tokens, the gate
decisions, and against the P0 run of the same request the first-token KL, whether
the greedy continuation is identical, and the share of it that agrees before the
first difference.  Outputs are compared as token lists (the synthetic streams have
no text).  `summarize` and `boot_ci` aggregate the rows into the report's fields
with the report's statistics (percentile bootstrap, 2000 resamples, seed 0).
"""

from __future__ import annotations

import time
from collections import Counter

import numpy as np


def boot_ci(x: np.ndarray, stat=np.mean, n: int = 2000, seed: int = 0) -> tuple[float, float]:
    """95 % percentile-bootstrap interval of `stat` over `x`.

    The published method that bench/report.py:17-22 uses: `n` resamples of len(x)
    indices drawn uniformly with replacement from numpy's default generator seeded
    with `seed`, the 2.5th and 97.5th percentiles of the resampled statistic.  All
    resamples are drawn as one (n, len(x)) index matrix (the generator yields the
    same index stream as one draw per resample) and the statistic is taken along
    its rows."""
    x = np.asarray(x)
    if x.size == 0:
        return float("nan"), float("nan")
    idx = np.random.default_rng(seed).integers(0, x.size, (n, x.size))
    samples = x[idx]
    try:
        stats = stat(samples, axis=1)
    except TypeError:  # a statistic without an axis argument
        stats = np.array([stat(row) for row in samples])
    lo, hi = np.percentile(stats, [2.5, 97.5])
    return float(lo), float(hi)


def _column(rows: list[dict], key: str, dtype=np.float64) -> np.ndarray:
    return np.fromiter((r[key] for r in rows), dtype=dtype, count=len(rows))


def summarize(rows: list[dict], skip_first: int = 0) -> dict:
    """One policy's replay rows -> the report fields of bench/report.py:29-57 that
    these replays produce: request count, TTFT p50 / p95, the token-weighted
    compute share, and, for rows compared with P0, the mean first-token KL and
    the share of outputs equal to P0's with its bootstrap interval; plus the
    counts of gate actions and reasons.  (The reference's accuracy, attack and
    conflict fields come from its labelled real-text traces; synthetic streams
    carry no such labels, so they are not summarised here.)"""
    rows = rows[skip_first:]
    ttft = _column(rows, "ttft")
    tokens = _column(rows, "tokens")
    p50, p95 = np.percentile(ttft, [50, 95])
    out = {"n": len(rows), "ttft_p50": float(p50), "ttft_p95": float(p95),
           "compute": float(np.sum(_column(rows, "compute") * tokens) / np.sum(tokens))}
    if rows and "kl" in rows[0]:
        match = _column(rows, "match_p0")
        out.update(kl=float(np.mean(_column(rows, "kl"))), match_p0=float(match.mean()),
                   match_ci=boot_ci(match))
    pairs = Counter((action, reason) for r in rows for action, reason in r["decisions"])
    actions, reasons = Counter(), Counter()
    for (action, reason), c in pairs.items():
        actions[action] += c
        reasons[reason] += c
    out["decisions"], out["reasons"] = dict(actions), dict(reasons)
    return out


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
