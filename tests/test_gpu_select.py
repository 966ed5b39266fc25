"""The pooled selection (torch_engine.py:125-153) on seeded random cases, against the oracle.

Each case draws a request of n_ctx positions and placements with random starts
(overlaps included), lengths, exact flags and per-chunk ratios, scores with many
exact ties (zero deviation is the common score of tokens whose fresh K/V equal the
cached ones), and optionally an escalation threshold placed between two chunks'
relative deviations.  Both device entry points must give exactly the oracle's kept
positions, budget, eligible count and recomputed-cached count:

  ckv_select_from_scores  - the selection alone, from given fp32 scores
  ckv_deviation_select    - phase 1 scores from K/V, then the same selection

n_ctx covers both homes of the per-position keys: the shared memory of the eight
CTAs of the selecting cluster (slices of up to 20128 positions, n_ctx <= 161024) and
the caller's scratch (above it).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from chunkkv_b200 import _lib, ops  # noqa: E402
from chunkkv_b200.engine.base import BlendConfig, plan_arrays  # noqa: E402
from oracle.blend_oracle import select  # noqa: E402

DEV = "cuda"
BF = torch.bfloat16


class _Chunk:
    def __init__(self, length):
        self.length = length


class _Place:
    def __init__(self, start, length, ratio, exact):
        self.start, self.ratio, self.exact, self.chunk = start, ratio, exact, _Chunk(length)


def _case(seed: int, n_ctx: int, n_chunks: int, overlap: bool, ties: float):
    rng = np.random.default_rng(seed)
    pl = []
    if overlap:
        for _ in range(n_chunks):
            ln = int(rng.integers(8, max(9, 2 * n_ctx // n_chunks)))
            st = int(rng.integers(0, n_ctx - ln))
            pl.append(_Place(st, ln, [None, 0.0, 0.3, 1.0][int(rng.integers(0, 4))], bool(rng.random() < 0.1)))
    else:
        bounds = np.sort(rng.choice(np.arange(1, n_ctx - 16), size=2 * n_chunks, replace=False))
        for c in range(n_chunks):
            st, en = int(bounds[2 * c]), int(bounds[2 * c + 1])
            pl.append(_Place(st, en - st, [None, None, 0.3, 0.0][int(rng.integers(0, 4))],
                             bool(rng.random() < 0.1)))
    cfg = BlendConfig(recompute_ratio=0.15, n_sink=4)
    plan = plan_arrays(n_ctx, pl, cfg.n_sink)
    diff = rng.random(n_ctx).astype(np.float32)
    diff[rng.random(n_ctx) < ties] = 0.0
    dup = rng.random(n_ctx) < 0.05
    diff[dup] = np.float32(0.25)  # a second block of exact ties
    norm = (rng.random(n_ctx) + 1.0).astype(np.float32)
    # positions never computed (exact) score 0 in the reference (zero-initialised
    # buffers, torch_engine.py:121-122); the kernel must ignore what the buffer holds there
    diff_ref, norm_ref = diff.copy(), norm.copy()
    diff_ref[plan.exact] = 0.0
    norm_ref[plan.exact] = 0.0
    diff[plan.exact] = 1e30
    norm[plan.exact] = 7.0
    return pl, cfg, plan, diff, norm, diff_ref, norm_ref


def _meta(pl, cfg):
    rows = []
    for p in pl:
        ratio = cfg.recompute_ratio if p.ratio is None else p.ratio
        rows.append([p.start, p.chunk.length, int(round(ratio * p.chunk.length)) if ratio > 0 else -1,
                     int(p.exact)])
    return torch.tensor(rows, dtype=torch.int32, device=DEV).reshape(-1, 4)


def _threshold(pl, diff_ref, norm_ref, rng):
    """A threshold halfway between two chunks' relative deviations (so fp32 summation
    order cannot flip a decision), or None."""
    rels = sorted({float(diff_ref[p.start:p.start + p.chunk.length].astype(np.float64).sum()
                         / norm_ref[p.start:p.start + p.chunk.length].astype(np.float64).sum())
                   for p in pl if not p.exact})
    if len(rels) < 2 or rng.random() < 0.4:
        return None
    i = int(rng.integers(0, len(rels) - 1))
    if rels[i + 1] - rels[i] < 1e-3 * max(1e-6, rels[i + 1]):
        return None
    return 0.5 * (rels[i] + rels[i + 1])


def _check(ws, pl, cfg, plan, diff_ref, norm_ref):
    n_ctx = plan.n
    ref = select(torch.from_numpy(diff_ref), torch.from_numpy(norm_ref), torch.from_numpy(plan.cached),
                 torch.from_numpy(plan.sink), pl, cfg)
    counts = ws.counts.cpu().numpy()
    keep = ref["keep_abs"].numpy()
    assert counts[0] == len(keep)
    np.testing.assert_array_equal(ws.keep_abs[:counts[0]].cpu().numpy(), keep)
    assert counts[2] == ref["budget"]
    assert counts[3] == int(ref["eligible"].sum())
    assert counts[1] == int(plan.cached[keep].sum())
    bad = bool(plan.exact[keep].any())
    assert bool(counts[5]) == bad
    if not bad:  # sel = each kept position's index among the non-exact positions
        active = np.flatnonzero(~plan.exact)
        np.testing.assert_array_equal(active[ws.sel[:counts[0]].cpu().numpy()], keep)
    rel = ws.rel[:len(pl)].cpu().numpy()
    got = rel[[not p.exact for p in pl]]
    want = np.array([c["rel_dev"] for c in ref["chunk_stats"]])
    np.testing.assert_allclose(got, want, rtol=2e-4)
    esc = [c["escalated"] for c in ref["chunk_stats"]]
    mask = 0
    for i, p in enumerate(pl[:32]):
        if not p.exact and esc[sum(1 for q in pl[:i] if not q.exact)]:
            mask |= 1 << i
    assert (int(counts[4]) & 0xffffffff) == mask
    return bad


CASES = [
    # seed, n_ctx, chunks, overlapping placements, share of zero scores
    (1, 300, 3, False, 0.5),
    (2, 5248, 10, False, 0.8),
    (3, 5248, 10, True, 0.3),
    (4, 161024, 300, False, 0.8),  # the largest n_ctx held in shared memory
    (5, 161025, 300, True, 0.5),   # the smallest in the caller's scratch
    (6, 32896, 64, False, 0.0),    # config 5's request length
    (7, 32896, 64, True, 0.9),
    (10, 20480, 40, False, 0.8),
    (8, 65536, 128, False, 0.6),
    (9, 1000, 200, True, 0.2),     # more chunks than warps in the CTA
    (11, 65536, 4096, False, 0.4),  # the largest chunk table
    (12, 37, 3, False, 0.5),       # fewer positions than CTAs x 16: empty slices
]


@pytest.mark.parametrize("seed,n_ctx,n_chunks,overlap,ties", CASES)
def test_select_from_scores_random_cases(seed, n_ctx, n_chunks, overlap, ties):
    rng = np.random.default_rng(100 + seed)
    pl, cfg, plan, diff, norm, diff_ref, norm_ref = _case(seed, n_ctx, n_chunks, overlap, ties)
    for thr in (None, _threshold(pl, diff_ref, norm_ref, rng)):
        cfg.escalate_threshold = thr
        ws = ops.SelectWorkspace(n_ctx, len(pl), DEV)
        ws.scratch.fill_(0xA5)  # the kernel must not depend on the scratch's old contents
        ops.select_from_scores(torch.from_numpy(diff).to(DEV), torch.from_numpy(norm).to(DEV),
                               torch.from_numpy(plan.pos_flags()).to(DEV), _meta(pl, cfg), thr, ws)
        bad = _check(ws, pl, cfg, plan, diff_ref, norm_ref)
        err = _lib.device_error()
        assert bool(err & 0x4) == bad


@pytest.mark.parametrize("n_ctx,n_chunks,H", [(5248, 10, 4), (32896, 64, 8)])
def test_deviation_select_fused_random_placements(n_ctx, n_chunks, H):
    """Phase 1 scores from K/V rows (cached everywhere except the query tail), then the
    selection: exact given the kernel's own scores, at the config-3 and config-5 lengths."""
    D = 128
    cl = (n_ctx - 128) // n_chunks
    rng = np.random.default_rng(n_ctx)
    order = rng.permutation(n_chunks)
    pl = [_Place(int(i) * cl, cl, None, False) for i in order]  # chunk table not in position order
    cfg = BlendConfig(recompute_ratio=0.15, n_sink=4)
    plan = plan_arrays(n_ctx, pl, cfg.n_sink)
    g = torch.Generator(device=DEV).manual_seed(n_ctx)
    Kb = torch.randn((H, n_ctx, D), generator=g, device=DEV).to(BF)
    Vb = torch.randn((H, n_ctx, D), generator=g, device=DEV).to(BF)
    kf = Kb.permute(1, 0, 2).reshape(n_ctx, H * D).clone()
    vf = Vb.permute(1, 0, 2).reshape(n_ctx, H * D).clone()
    noisy = torch.rand(n_ctx, generator=g, device=DEV) < 0.2
    kf[noisy] = (kf[noisy].float() + 0.05 * torch.randn(kf[noisy].shape, generator=g, device=DEV)).to(BF)
    vf[noisy] = (vf[noisy].float() + 0.05 * torch.randn(vf[noisy].shape, generator=g, device=DEV)).to(BF)
    active = torch.arange(n_ctx, dtype=torch.int32, device=DEV)
    ws = ops.SelectWorkspace(n_ctx, len(pl), DEV)
    for _ in range(2):  # the ticket counter and scratch are reused by the second launch
        ops.deviation_select(kf, vf, Kb, Vb, active, torch.from_numpy(plan.pos_flags()).to(DEV), _meta(pl, cfg),
                             None, ws)
        _check(ws, pl, cfg, plan, ws.diff[:n_ctx].cpu().numpy(), ws.norm[:n_ctx].cpu().numpy())
    assert not ws.control.any()  # ticket and histogram back at zero
    # phase 1 against the formula of torch_engine.py:118-120 (zero base where nothing is cached)
    kr = kf.view(n_ctx, H, D).permute(1, 0, 2)
    vr = vf.view(n_ctx, H, D).permute(1, 0, 2)
    cm = torch.from_numpy(plan.cached).to(DEV)[None, :, None]
    Kz, Vz = torch.where(cm, Kb, torch.zeros_like(Kb)), torch.where(cm, Vb, torch.zeros_like(Vb))
    d_ref = ((kr - Kz).float() ** 2).sum(dim=(0, 2)) + ((vr - Vz).float() ** 2).sum(dim=(0, 2))
    n_ref = (kr.float() ** 2).sum(dim=(0, 2)) + (vr.float() ** 2).sum(dim=(0, 2))
    torch.testing.assert_close(ws.diff[:n_ctx], d_ref, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(ws.norm[:n_ctx], n_ref, rtol=1e-4, atol=1e-4)
    assert _lib.device_error() == 0
