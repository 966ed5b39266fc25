"""Each CUDA kernel against a plain torch statement of the same op (run on the GPU
in fp32 where the op is floating point), or against the oracle for the selection.

Tolerances: bf16 outputs must match within max |err| / max |ref| <= 1e-2 (the
north-star bf16 tolerance); ops whose reference rounding points we reproduce
exactly are also checked for (near-)bitwise agreement.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

from chunkkv_b200 import _lib, ops  # noqa: E402

DEV = "cuda"
BF = torch.bfloat16


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def row_rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """Worst row of max |a - b| / max |b| over the last dimension, so that rows of small
    magnitude are held to the same relative bar as the largest ones."""
    a, b = a.float().flatten(0, -2), b.float().flatten(0, -2)
    return float(((a - b).abs().amax(-1) / b.abs().amax(-1).clamp_min(1e-30)).max())


def inv_freq(D, theta=1e6, device=DEV):
    return theta ** (-torch.arange(0, D, 2, device=device, dtype=torch.float32) / D)


def torch_rotate(x, angles):
    """TorchEngine._rotate (torch_engine.py:46-51) restated."""
    cos, sin = angles.cos(), angles.sin()
    half = x.shape[-1] // 2
    x32 = x.float()
    x1, x2 = x32[..., :half], x32[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).to(x.dtype)


@pytest.fixture(autouse=True)
def _device_error_free():
    yield
    _lib.check_device()


# ------------------------------------------------------------------ re-RoPE
@pytest.mark.parametrize("D", [64, 128])
def test_rope_table_matches_torch(D):
    inv = inv_freq(D)
    tab = ops.rope_table(inv, 5000)
    ang = torch.arange(5000, device=DEV).float()[:, None] * inv[None, :]
    assert torch.equal(tab[..., 0], ang.cos()) or (tab[..., 0] - ang.cos()).abs().max() < 1e-6
    assert (tab[..., 1] - ang.sin()).abs().max() < 1e-6


@pytest.mark.parametrize("D,delta", [(64, 37), (128, -4096), (128, 4095), (64, 16384), (256, 1234)])
def test_shift_keys_matches_reference_rotation(D, delta):
    """Head dims 64 / 128 take one fill of a warp's 4 KiB staging slot per 16-row unit, 256 takes
    two (8 rows each)."""
    g = torch.Generator(device=DEV).manual_seed(1)
    k = torch.randn((1, 4, 300, D), generator=g, device=DEV).to(BF)
    inv = inv_freq(D)
    ref = torch_rotate(k, (delta * inv)[None, :].expand(k.shape[-2], -1))
    out = ops.shift_keys(k, delta, inv)
    assert rel_err(out, ref) <= 1e-2
    # same rounding points as the reference: at most a last-bit difference from cos/sin
    assert (out.float() != ref.float()).float().mean() < 1e-3


def test_shift_round_trip_and_compose():
    """rerope tests (test_rerope.py:20-27): shift(rope(x,5),37) == rope(x,42); +-37 round trip."""
    from chunkkv_b200.scheduler.rerope import RopeSpec, apply_rope, shift_keys

    spec = RopeSpec(dims=64, base=1e6)
    x = torch.randn((1, 2, 10, 64), device=DEV).to(BF)
    at5 = apply_rope(x, torch.arange(5, 15, device=DEV), spec)
    at42 = apply_rope(x, torch.arange(42, 52, device=DEV), spec)
    assert rel_err(shift_keys(at5, 37, spec), at42) <= 1e-2
    back = shift_keys(shift_keys(at5, 37, spec), -37, spec)
    assert rel_err(back, at5) <= 1e-2
    assert shift_keys(at5, 0, spec) is at5


def test_apply_rope_matches_reference_rope():
    D = 128
    x = torch.randn((2, 3, 77, D), device=DEV).to(BF)
    pos = torch.randperm(9000, device=DEV)[:77].sort().values
    inv = inv_freq(D)
    ref = torch_rotate(x, pos.float()[:, None] * inv[None, :])
    out = ops.apply_rope(x, pos, inv)
    assert rel_err(out, ref) <= 1e-2
    assert (out.float() != ref.float()).float().mean() < 1e-3


@pytest.mark.parametrize("D", [64, 128, 256])
def test_fp32_keys_stay_fp32(D):
    """The reference rotates in fp32 and returns the input dtype (torch_engine.py:46-51,
    56-59; rerope.py:36-61): fp32 keys come back fp32, rotated with fp32 rounding.  The
    only difference from the torch restatement is the ulp of cos/sin, so the bar is
    fp32-sized: max |err| <= 4e-6 x max |ref|."""
    from chunkkv_b200.scheduler import rerope

    g = torch.Generator(device=DEV).manual_seed(5)
    k = torch.randn((1, 4, 300, D), generator=g, device=DEV)
    inv = inv_freq(D)
    for delta in (1, -37, 4096, -16384):
        ref = torch_rotate(k, (delta * inv)[None, :].expand(k.shape[-2], -1))
        out = ops.shift_keys(k, delta, inv)
        assert out.dtype == torch.float32 and rel_err(out, ref) <= 4e-6, delta
    pos = torch.randperm(30000, device=DEV)[:300].sort().values
    ref = torch_rotate(k, pos.float()[:, None] * inv[None, :])
    out = ops.apply_rope(k, pos, inv)
    assert out.dtype == torch.float32 and rel_err(out, ref) <= 4e-6
    # the scheduler API (RopeSpec) keeps the dtype of its input too
    spec = rerope.RopeSpec(dims=D, base=1e6)
    sk = rerope.shift_keys(k, 77, spec)
    assert sk.dtype == torch.float32
    assert rel_err(sk, torch_rotate(k, (77 * inv)[None, :].expand(k.shape[-2], -1))) <= 4e-6
    kb = k.to(BF)
    assert rerope.shift_keys(kb, 77, spec).dtype == BF and rerope.apply_rope(kb, pos, spec).dtype == BF
    assert rerope.apply_rope(k, pos, spec).dtype == torch.float32
    # a round trip in fp32 returns the keys to fp32 accuracy
    back = ops.shift_keys(ops.shift_keys(k, 1234, inv), -1234, inv)
    assert rel_err(back, k) <= 1e-5
    with pytest.raises(NotImplementedError):
        ops.shift_keys(k.half(), 3, inv)


def test_engine_shift_keys_keeps_dtype():
    """TorchEngine.shift_keys (torch_engine.py:56-59) returns the input dtype."""
    from chunkkv_b200.engine.torch_engine import TorchEngine
    from chunkkv_b200.engine.weights import SHAPES, random_packed

    eng = TorchEngine.from_packed(random_packed(SHAPES["tiny"], seed=0, device=DEV))
    k32 = torch.randn((1, eng.n_kv, 50, eng.head_dim), device=DEV)
    out = eng.shift_keys(k32, 11)
    assert out.dtype == torch.float32
    ref = torch_rotate(k32, (11 * eng.inv_freq)[None, :].expand(50, -1))
    assert rel_err(out, ref) <= 4e-6
    assert eng.shift_keys(k32.to(BF), 11).dtype == BF
    with pytest.raises(NotImplementedError):
        eng.shift_keys(k32.half(), 11)


def test_partial_rotary_dims_copy_tail():
    D, rot = 128, 64
    x = torch.randn((1, 2, 40, D), device=DEV).to(BF)
    inv = 1e6 ** (-torch.arange(0, rot // 2, device=DEV, dtype=torch.float32) * 2.0 / rot)
    out = ops.shift_keys(x, 11, inv, rot_dims=rot)
    ref = torch_rotate(x[..., :rot], (11 * inv)[None, :].expand(40, -1))
    assert rel_err(out[..., :rot], ref) <= 1e-2
    assert torch.equal(out[..., rot:], x[..., rot:])


# ---------------------------------------------------------- gather / pages
def _make_pool(L, H, D, n_pages, seed=0):
    from chunkkv_b200.store.pages import PagePool

    pool = PagePool(L, H, D, n_pages, DEV)
    g = torch.Generator(device=DEV).manual_seed(seed)
    pool.pages.copy_(torch.randn(pool.pages.shape, generator=g, device=DEV).to(BF))
    return pool


def _chunk_dense(pool, ids, length, src_off=0):
    """Per-layer dense K/V of a paged chunk, read with torch indexing."""
    pg = pool.pages[torch.as_tensor(ids, device=DEV).long()]      # [n, L, 2, H, 16, D]
    t = pg.permute(1, 2, 3, 0, 4, 5).reshape(pool.n_layers, 2, pool.n_kv_heads, -1, pool.head_dim)
    return t[:, 0, :, src_off:src_off + length], t[:, 1, :, src_off:src_off + length]


@pytest.mark.parametrize("L,H,D", [(3, 4, 128), (4, 2, 64), (2, 2, 256)])
def test_blend_gather_paged(L, H, D):
    pool = _make_pool(L, H, D, 64)
    rng = np.random.default_rng(0)
    N = 700
    chunks = [  # (length, dst_start, src_start, layer_begin, src_offset)
        (100, 10, 400, 1, 0), (37, 150, 0, 0, 5), (256, 200, 1000, 1, 0), (16, 600, 600, 0, 0)]
    table, meta = [], []
    for length, dst, src, lb, off in chunks:
        n = (length + off + 15) // 16
        ids = rng.choice(64, size=n, replace=False).astype(np.int32)
        meta.append([len(table), length, dst, dst - src, lb, L, off, 0])
        table.extend(ids.tolist())
    inv = inv_freq(D)
    k_out = torch.zeros((L, H, N, D), dtype=BF, device=DEV)
    v_out = torch.zeros_like(k_out)
    ops.blend_gather_paged(pool.pages, torch.tensor(table, dtype=torch.int32, device=DEV),
                           torch.tensor(meta, dtype=torch.int32, device=DEV), inv, k_out, v_out, 0, L)
    k_ref = torch.zeros_like(k_out)
    v_ref = torch.zeros_like(v_out)
    for (length, dst, src, lb, off), m in zip(chunks, meta):
        ids = table[m[0]:m[0] + (length + off + 15) // 16]
        kd, vd = _chunk_dense(pool, ids, length, off)
        delta = dst - src
        for li in range(lb, L):
            kk = kd[li] if delta == 0 else torch_rotate(kd[li], (delta * inv)[None, :].expand(length, -1))
            k_ref[li, :, dst:dst + length] = kk
            v_ref[li, :, dst:dst + length] = vd[li]
    assert torch.equal(v_out, v_ref)
    assert rel_err(k_out, k_ref) <= 1e-2
    assert (k_out.float() != k_ref.float()).float().mean() < 1e-3


@pytest.mark.parametrize("D", [64, 128, 256])
def test_blend_gather_dense_and_pages_roundtrip(D):
    L, H, length = 3, 4, 77
    from chunkkv_b200.store.pages import PagedChunkKV, PagePool

    pool = PagePool(L, H, D, 16, DEV)
    ks = [torch.randn((1, H, length, D), device=DEV).to(BF) for _ in range(L)]
    vs = [torch.randn((1, H, length, D), device=DEV).to(BF) for _ in range(L)]
    ids = pool.alloc((length + 15) // 16)
    pool.write(ids, length, ks, vs)
    c = PagedChunkKV(pool, ids, length, start=0)
    for li in range(L):
        assert torch.equal(c.keys[li], ks[li]) and torch.equal(c.values[li], vs[li])
    # dense gather of the same chunk with a shift
    N, dst, delta = 200, 50, 50
    inv = inv_freq(D)
    kp = torch.tensor([k.data_ptr() for k in ks], dtype=torch.uint64, device=DEV)
    vp = torch.tensor([v.data_ptr() for v in vs], dtype=torch.uint64, device=DEV)
    meta = torch.tensor([[0, length, dst, delta, 0, L, 0, ks[0].stride(1)]], dtype=torch.int32, device=DEV)
    k_out = torch.zeros((L, H, N, D), dtype=BF, device=DEV)
    v_out = torch.zeros_like(k_out)
    ops.blend_gather_dense(kp, vp, meta, inv, k_out, v_out, 0, L)
    for li in range(L):
        ref = torch_rotate(ks[li][0], (delta * inv)[None, :].expand(length, -1))
        assert rel_err(k_out[li, :, dst:dst + length], ref) <= 1e-2
        assert torch.equal(v_out[li, :, dst:dst + length], vs[li][0])


def test_page_id_out_of_range_is_reported_not_faulted():
    pool = _make_pool(2, 2, 64, 4)
    meta = torch.tensor([[0, 16, 0, 0, 0, 2, 0, 0]], dtype=torch.int32, device=DEV)
    table = torch.tensor([99], dtype=torch.int32, device=DEV)  # outside the pool: skipped by the kernel
    k = torch.zeros((2, 2, 16, 64), dtype=BF, device=DEV)
    ops.blend_gather_paged(pool.pages, table, meta, inv_freq(64), k, k.clone(), 0, 2)
    assert _lib.device_error() & 0x2


# --------------------------------------------------------------- selection
def _sel_meta(place, chunk_len, cfg):
    rows = []
    for p in place:
        ratio = cfg.recompute_ratio if p["ratio"] is None else p["ratio"]
        rows.append([p["start"], chunk_len, int(round(ratio * chunk_len)) if ratio > 0 else -1, int(p["exact"])])
    return torch.tensor(rows, dtype=torch.int32, device=DEV).reshape(-1, 4)


@pytest.mark.parametrize("name", ["tiny_fp32", "tiny_escalate", "tiny_exact_overflow", "tiny7_fp32",
                                  "cfg1_0p5b"])
def test_select_from_reference_scores_is_bit_exact(name):
    """Given the reference's own fp32 layer-1 scores, the kernel keeps exactly its tokens."""
    from chunkkv_b200.engine.base import plan_arrays
    from helpers import scenario
    from scenarios import SCENARIOS

    s = scenario(name)
    a = s.arrays
    L = SCENARIOS[name].chunk_len
    N = len(s.tokens)

    class C:
        length = L

    class P:
        def __init__(self, p):
            self.start, self.ratio, self.exact, self.chunk = p["start"], p["ratio"], p["exact"], C()

    plan = plan_arrays(N, [P(p) for p in s.place], s.config.n_sink)
    ws = ops.SelectWorkspace(N, len(s.place), DEV)
    ops.select_from_scores(torch.from_numpy(a["diff"]).to(DEV), torch.from_numpy(a["norm"]).to(DEV),
                           torch.from_numpy(plan.pos_flags()).to(DEV), _sel_meta(s.place, L, s.config),
                           s.config.escalate_threshold, ws)
    counts = ws.counts.cpu().numpy()
    n_sel = counts[0]
    np.testing.assert_array_equal(ws.keep_abs[:n_sel].cpu().numpy(), a["keep_abs"])
    assert counts[2] == s.meta["budget"]
    assert counts[1] == s.meta["stats"]["recomputed_cached_tokens"]
    rel = ws.rel[:len(s.place)].cpu().numpy()
    ref_rel = [c["rel_dev"] for c in s.meta["stats"]["chunks"]]
    np.testing.assert_allclose(rel[[not p["exact"] for p in s.place]], ref_rel, rtol=1e-5)
    # sel = index of each kept position among the non-exact (layer-1 active) positions
    active = np.flatnonzero(~plan.exact)
    np.testing.assert_array_equal(active[ws.sel[:n_sel].cpu().numpy()], a["keep_abs"])


def test_select_ties_lower_position_first_and_microbench_shape():
    """Config-2 shape: 8 x 256 chunks, exact-zero deviation on 80 % of tokens."""
    from chunkkv_b200.engine.base import BlendConfig
    from oracle.blend_oracle import select

    g = torch.Generator().manual_seed(2)
    N, n_ch, cl = 2048, 8, 256
    diff = torch.zeros(N)
    noisy = torch.rand(N, generator=g) < 0.2
    diff[noisy] = torch.rand(int(noisy.sum()), generator=g) + 0.01
    diff[100:104] = 0.5  # an exact tie straddling the threshold region
    norm = torch.rand(N, generator=g) + 1.0
    cfg = BlendConfig(recompute_ratio=0.15, n_sink=4)

    class C:
        length = cl

    class P:
        def __init__(self, s):
            self.start, self.ratio, self.exact, self.chunk = s, None, False, C()

    pl = [P(i * cl) for i in range(n_ch)]
    cached = torch.ones(N, dtype=torch.bool)
    sink = torch.zeros(N, dtype=torch.bool)
    for p in pl:
        sink[p.start:p.start + 4] = True
    ref = select(diff, norm, cached, sink, pl, cfg)
    flags = (cached.to(torch.uint8) | (sink.to(torch.uint8) << 1)).to(DEV)
    meta = torch.tensor([[p.start, cl, 38, 0] for p in pl], dtype=torch.int32, device=DEV)
    ws = ops.SelectWorkspace(N, n_ch, DEV)
    ops.select_from_scores(diff.to(DEV), norm.to(DEV), flags, meta, None, ws)
    n_sel = int(ws.counts[0])
    assert n_sel == 304 + 32
    np.testing.assert_array_equal(ws.keep_abs[:n_sel].cpu().numpy(), ref["keep_abs"].numpy())


def test_deviation_select_fused_matches_formula_and_selection():
    from oracle.blend_oracle import select
    from chunkkv_b200.engine.base import BlendConfig

    H, D, N, n_ch, cl = 4, 128, 2048 + 64, 8, 256
    g = torch.Generator(device=DEV).manual_seed(3)
    Kb = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    Vb = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    active = torch.arange(N, dtype=torch.int32, device=DEV)
    kf = Kb.permute(1, 0, 2).reshape(N, H * D).clone()
    vf = Vb.permute(1, 0, 2).reshape(N, H * D).clone()
    noisy = torch.rand(N, generator=g, device=DEV) < 0.2
    kf[noisy] = (kf[noisy].float() + 0.05 * torch.randn(kf[noisy].shape, generator=g, device=DEV)).to(BF)
    vf[noisy] = (vf[noisy].float() + 0.05 * torch.randn(vf[noisy].shape, generator=g, device=DEV)).to(BF)
    # fresh query tail (not cached)
    cached = torch.zeros(N, dtype=torch.bool)
    cached[:n_ch * cl] = True
    sink = torch.zeros(N, dtype=torch.bool)
    for c in range(n_ch):
        sink[c * cl:c * cl + 4] = True
    flags = (cached.to(torch.uint8) | (sink.to(torch.uint8) << 1)).to(DEV)
    meta = torch.tensor([[c * cl, cl, 38, 0] for c in range(n_ch)], dtype=torch.int32, device=DEV)
    ws = ops.SelectWorkspace(N, n_ch, DEV)
    ops.deviation_select(kf, vf, Kb, Vb, active, flags, meta, None, ws)
    # formula of torch_engine.py:118-120 on the same data; the reference's base cache is
    # zero wherever no chunk was placed (torch_engine.py:97), i.e. at the fresh query tail
    kr = kf.view(N, H, D).permute(1, 0, 2)
    vr = vf.view(N, H, D).permute(1, 0, 2)
    cm = cached.to(DEV)[None, :, None]
    Kz, Vz = torch.where(cm, Kb, torch.zeros_like(Kb)), torch.where(cm, Vb, torch.zeros_like(Vb))
    d_ref = ((kr - Kz).float() ** 2).sum(dim=(0, 2)) + ((vr - Vz).float() ** 2).sum(dim=(0, 2))
    n_ref = (kr.float() ** 2).sum(dim=(0, 2)) + (vr.float() ** 2).sum(dim=(0, 2))
    torch.testing.assert_close(ws.diff[:N], d_ref, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(ws.norm[:N], n_ref, rtol=1e-4, atol=1e-4)
    # selection is exact given the kernel's own scores

    class C:
        length = cl

    class P:
        def __init__(self, s):
            self.start, self.ratio, self.exact, self.chunk = s, None, False, C()

    ref = select(ws.diff[:N].cpu(), ws.norm[:N].cpu(), cached, sink, [P(c * cl) for c in range(n_ch)],
                 BlendConfig(recompute_ratio=0.15, n_sink=4))
    n_sel = int(ws.counts[0])
    np.testing.assert_array_equal(ws.keep_abs[:n_sel].cpu().numpy(), ref["keep_abs"].numpy())
    # the ticket counter is back at zero: a second launch works the same
    ops.deviation_select(kf, vf, Kb, Vb, active, flags, meta, None, ws)
    assert int(ws.counts[0]) == n_sel and not ws.control.any()
    # scores only, per head group (tensor-parallel ranks): the group sums are the fused
    # kernel's scores, and the selection from them is the fused kernel's selection
    parts = []
    for hs in (slice(0, 2), slice(2, 4)):
        w2 = ops.SelectWorkspace(N, n_ch, DEV)
        cols = slice(hs.start * D, hs.stop * D)
        ops.deviation_scores(kf[:, cols].contiguous(), vf[:, cols].contiguous(), Kb[hs].contiguous(),
                             Vb[hs].contiguous(), active, flags, w2)
        parts.append(w2.scores.clone())
    tot = parts[0] + parts[1]
    torch.testing.assert_close(tot[0, :N], ws.diff[:N], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(tot[1, :N], ws.norm[:N], rtol=1e-5, atol=1e-4)
    w3 = ops.SelectWorkspace(N, n_ch, DEV)
    w3.scores.copy_(tot)
    ops.select_from_scores(w3.diff[:N], w3.norm[:N], flags, meta, None, w3)
    ref3 = select(w3.diff[:N].cpu(), w3.norm[:N].cpu(), cached, sink, [P(c * cl) for c in range(n_ch)],
                  BlendConfig(recompute_ratio=0.15, n_sink=4))
    n3 = int(w3.counts[0])
    np.testing.assert_array_equal(w3.keep_abs[:n3].cpu().numpy(), ref3["keep_abs"].numpy())


# ------------------------------------------------------------------- GEMMs
GEMM_SHAPES = [(1, 256, 256), (100, 896, 896), (938, 4608, 3584), (1000, 512, 1152), (257, 3584, 18944)]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
def test_linear_matches_fp32(m, n, k):
    g = torch.Generator(device=DEV).manual_seed(m + n)
    x = torch.randn((m, k), generator=g, device=DEV).to(BF)
    w = (torch.randn((n, k), generator=g, device=DEV) * 0.02).to(BF)
    b = (torch.randn(n, generator=g, device=DEV) * 0.02).to(BF)
    out = ops.linear(x, w, b)
    ref = x.float() @ w.float().T + b.float()
    assert rel_err(out, ref) <= 1e-2
    out_nb = ops.linear(x, w)
    assert rel_err(out_nb, x.float() @ w.float().T) <= 1e-2


def test_linear_many_tiles_persistent_loop():
    """More tiles than SMs: every tile of the persistent schedule is written."""
    m, n, k = 4096, 4096, 512
    x = torch.randn((m, k), device=DEV).to(BF)
    w = (torch.randn((n, k), device=DEV) * 0.05).to(BF)
    out = ops.linear(x, w)
    assert rel_err(out, x.float() @ w.float().T) <= 1e-2


@pytest.mark.parametrize("m,n", [(938, 3584), (938, 3648), (1024, 896)])
def test_linear_residual_narrow_tiles(m, n):
    """Shapes whose makespan is shorter with 224-column tiles (incl. a ragged last tile)."""
    k = 1152
    g = torch.Generator(device=DEV).manual_seed(m * n)
    a = torch.randn((m, k), generator=g, device=DEV).to(BF)
    w = (torch.randn((n, k), generator=g, device=DEV) * 0.02).to(BF)
    h = torch.randn((m, n), generator=g, device=DEV).to(BF)
    ref = h.float() + (a.float() @ w.float().T).to(BF).float()
    ops.linear_residual(a, w, h)
    assert rel_err(h, ref) <= 1e-2
    out = ops.linear(a, w)
    assert rel_err(out, a.float() @ w.float().T) <= 1e-2


def test_linear_residual_and_swiglu():
    from chunkkv_b200.engine.weights import interleave_gate_up

    m, hid, inter = 333, 896, 1024
    x = torch.randn((m, hid), device=DEV).to(BF)
    w = (torch.randn((hid, inter), device=DEV) * 0.02).to(BF)
    a = torch.randn((m, inter), device=DEV).to(BF)
    h = torch.randn((m, hid), device=DEV).to(BF)
    ref = (h.float() + (a.float() @ w.float().T).to(BF).float())
    ops.linear_residual(a, w, h)
    assert rel_err(h, ref) <= 1e-2
    wg = (torch.randn((inter, hid), device=DEV) * 0.02).to(BF)
    wu = (torch.randn((inter, hid), device=DEV) * 0.02).to(BF)
    out = torch.empty((m, inter), dtype=BF, device=DEV)
    ops.linear_swiglu(x, interleave_gate_up(wg, wu), out)
    gg = (x.float() @ wg.float().T).to(BF)
    uu = (x.float() @ wu.float().T).to(BF)
    ref2 = (F.silu(gg) * uu).float()
    assert rel_err(out, ref2) <= 1e-2


@pytest.mark.parametrize("m,hid", [(1, 3584), (2, 896), (4, 5120)])
def test_decode_gemv_fused_rmsnorm_matches_rmsnorm_then_gemv(m, hid):
    """ckv_gemv_swiglu_rmsnorm / ckv_gemv_qkv_rope_rmsnorm (each CTA normalises h itself)
    against ckv_rmsnorm followed by the plain GEMVs: the same rounding points, so they may
    differ only where the sum of squares, added in another order, moves the scale."""
    from chunkkv_b200.engine.weights import interleave_gate_up

    inter, Hq, H, D, N = 1024, 8, 2, 128, 300
    g = torch.Generator(device=DEV).manual_seed(hid + m)
    h = torch.randn((m, hid), generator=g, device=DEV).to(BF)
    lnw = (1 + 0.1 * torch.randn(hid, generator=g, device=DEV)).to(BF)
    x = ops.rmsnorm(h, lnw, 1e-6)
    wgu = interleave_gate_up((torch.randn((inter, hid), generator=g, device=DEV) * 0.02).to(BF),
                             (torch.randn((inter, hid), generator=g, device=DEV) * 0.02).to(BF))
    o1, o2 = (torch.empty((m, inter), dtype=BF, device=DEV) for _ in range(2))
    ops.gemv_swiglu(h, wgu, o1, norm_w=lnw, eps=1e-6)
    ops.gemv_swiglu(x, wgu, o2)
    assert rel_err(o1, o2) <= 1e-2
    assert (o1 != o2).float().mean() < 0.02
    cols = (Hq + 2 * H) * D
    wq = (torch.randn((cols, hid), generator=g, device=DEV) * 0.05).to(BF)
    bq = (torch.randn(cols, generator=g, device=DEV) * 0.05).to(BF)
    pos = torch.randperm(N, generator=g, device=DEV)[:m].sort().values.to(torch.int32)
    tab = ops.rope_table(inv_freq(D), 512)
    q1, q2 = (torch.empty((m, Hq * D), dtype=BF, device=DEV) for _ in range(2))
    K1, V1, K2, V2 = (torch.zeros((H, N, D), dtype=BF, device=DEV) for _ in range(4))
    ops.gemv_qkv_rope(h, wq, bq, Hq, H, D, pos, tab, q1, K1, V1, norm_w=lnw, eps=1e-6)
    ops.gemv_qkv_rope(x, wq, bq, Hq, H, D, pos, tab, q2, K2, V2)
    assert rel_err(q1, q2) <= 1e-2 and (q1 != q2).float().mean() < 0.02
    assert rel_err(K1, K2) <= 1e-2 and rel_err(V1, V2) <= 1e-2


@pytest.mark.parametrize("m,k", [(1, 9472), (3, 18944)])
def test_decode_gemv_residual_long_rows(m, k):
    """Long rows (k >= 8192: four warps per row, partial sums through shared memory) against
    the tcgen05 residual GEMM and an fp32 reference."""
    g = torch.Generator(device=DEV).manual_seed(k + m)
    a = torch.randn((m, k), generator=g, device=DEV).to(BF)
    for n in (528, 517):  # 517: the last CTA's second row is past n
        w = (torch.randn((n, k), generator=g, device=DEV) * 0.02).to(BF)
        h = torch.randn((m, n), generator=g, device=DEV).to(BF)
        h1 = h.clone()
        ops.gemv_residual(a, w, h1)
        ref = h.float() + (a.float() @ w.float().T).to(BF).float()
        assert rel_err(h1, ref) <= 1e-2
        if n % 16 == 0:  # the GEMM path takes multiples of 16
            h2 = h.clone()
            ops.linear_residual(a, w, h2)
            assert rel_err(h1, h2) <= 1e-2


@pytest.mark.parametrize("m", [1, 3, 8])
def test_decode_gemv_epilogues_match_the_gemm_path(m):
    """ckv_gemv_residual / _swiglu / _qkv_rope (m <= 8) against the tcgen05 GEMM entry points
    with the same epilogues, and against fp32 references."""
    from chunkkv_b200.engine.weights import interleave_gate_up

    hid, inter, Hq, H, D, N = 896, 1024, 7, 1, 128, 300
    g = torch.Generator(device=DEV).manual_seed(m)
    x = torch.randn((m, hid), generator=g, device=DEV).to(BF)
    a = torch.randn((m, inter), generator=g, device=DEV).to(BF)
    w = (torch.randn((hid, inter), generator=g, device=DEV) * 0.02).to(BF)
    h = torch.randn((m, hid), generator=g, device=DEV).to(BF)
    h1, h2 = h.clone(), h.clone()
    ops.gemv_residual(a, w, h1)
    ops.linear_residual(a, w, h2)
    ref = h.float() + (a.float() @ w.float().T).to(BF).float()
    assert rel_err(h1, ref) <= 1e-2 and rel_err(h1, h2) <= 1e-2
    wg = (torch.randn((inter, hid), generator=g, device=DEV) * 0.02).to(BF)
    wu = (torch.randn((inter, hid), generator=g, device=DEV) * 0.02).to(BF)
    wgu = interleave_gate_up(wg, wu)
    o1 = torch.empty((m, inter), dtype=BF, device=DEV)
    o2 = torch.empty_like(o1)
    ops.gemv_swiglu(x, wgu, o1)
    ops.linear_swiglu(x, wgu, o2)
    ref2 = (F.silu((x.float() @ wg.float().T).to(BF)) * (x.float() @ wu.float().T).to(BF)).float()
    assert rel_err(o1, ref2) <= 1e-2 and rel_err(o1, o2) <= 1e-2
    cols = (Hq + 2 * H) * D
    wq = (torch.randn((cols, hid), generator=g, device=DEV) * 0.05).to(BF)
    bq = (torch.randn(cols, generator=g, device=DEV) * 0.05).to(BF)
    pos = torch.randperm(N, generator=g, device=DEV)[:m].sort().values.to(torch.int32)
    tab = ops.rope_table(inv_freq(D), 512)
    q1, q2 = torch.empty((m, Hq * D), dtype=BF, device=DEV), torch.empty((m, Hq * D), dtype=BF, device=DEV)
    K1, V1 = torch.zeros((H, N, D), dtype=BF, device=DEV), torch.zeros((H, N, D), dtype=BF, device=DEV)
    K2, V2 = K1.clone(), V1.clone()
    ops.gemv_qkv_rope(x, wq, bq, Hq, H, D, pos, tab, q1, K1, V1)
    ops.qkv_rope(x, wq, bq, m, 0, cols, Hq, H, D, pos, tab, q_out=q2, k_cache=K2, v_cache=V2)
    assert rel_err(q1, q2) <= 1e-2
    assert rel_err(K1[:, pos.long()], K2[:, pos.long()]) <= 1e-2
    assert rel_err(V1[:, pos.long()], V2[:, pos.long()]) <= 1e-2


@pytest.mark.parametrize("Hq,H,D,hid", [(28, 4, 128, 512), (14, 2, 64, 896), (4, 2, 64, 256),
                                        (5, 1, 128, 5120)])
def test_qkv_rope_scatter_and_compact(Hq, H, D, hid):
    m, N = 300, 1000
    g = torch.Generator(device=DEV).manual_seed(Hq)
    x = torch.randn((m, hid), generator=g, device=DEV).to(BF)
    cols = (Hq + 2 * H) * D
    w = (torch.randn((cols, hid), generator=g, device=DEV) * 0.05).to(BF)
    b = (torch.randn(cols, generator=g, device=DEV) * 0.05).to(BF)
    pos = torch.randperm(N, generator=g, device=DEV)[:m].sort().values.to(torch.int32)
    inv = inv_freq(D)
    tab = ops.rope_table(inv, 4096)
    q = torch.empty((m, Hq * D), dtype=BF, device=DEV)
    Kc = torch.zeros((H, N, D), dtype=BF, device=DEV)
    Vc = torch.zeros_like(Kc)
    ops.qkv_rope(x, w, b, m, 0, cols, Hq, H, D, pos, tab, q_out=q, k_cache=Kc, v_cache=Vc)
    y = (x.float() @ w.float().T + b.float()).to(BF)
    qr = y[:, :Hq * D].view(m, Hq, D).transpose(0, 1)
    kr = y[:, Hq * D:(Hq + H) * D].view(m, H, D).transpose(0, 1)
    vr = y[:, (Hq + H) * D:].view(m, H, D).transpose(0, 1)
    ang = pos.float()[:, None] * inv[None, :]
    q_ref = torch_rotate(qr, ang).transpose(0, 1).reshape(m, Hq * D)
    k_ref = torch_rotate(kr, ang)
    assert rel_err(q, q_ref) <= 1e-2
    assert rel_err(Kc[:, pos.long()], k_ref) <= 1e-2
    assert rel_err(Vc[:, pos.long()], vr) <= 1e-2
    # compact k/v for the K/V columns only (the layer-1 deviation input)
    kc = torch.empty((m, H * D), dtype=BF, device=DEV)
    vc = torch.empty_like(kc)
    ops.qkv_rope(x, w, b, m, Hq * D, cols, Hq, H, D, pos, tab, k_compact=kc, v_compact=vc)
    assert rel_err(kc.view(m, H, D).transpose(0, 1), k_ref) <= 1e-2
    assert rel_err(vc.view(m, H, D).transpose(0, 1), vr) <= 1e-2


# --------------------------------------------------------------- attention
@pytest.mark.parametrize("Hq,H,D,N,m", [(28, 4, 128, 1500, 300), (14, 2, 64, 700, 700), (4, 2, 64, 100, 37),
                                        (7, 1, 128, 4100, 1), (14, 2, 64, 700, 1), (16, 1, 128, 3000, 1),
                                        (20, 1, 64, 500, 1), (10, 2, 128, 900, 1), (16, 2, 64, 600, 1),
                                        (6, 6, 64, 300, 1)])
def test_attention_matches_masked_sdpa(Hq, H, D, N, m):
    g = torch.Generator(device=DEV).manual_seed(N)
    q = torch.randn((m, Hq, D), generator=g, device=DEV).to(BF)
    K = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    V = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    if m == N:
        pos = torch.arange(N, device=DEV, dtype=torch.int32)
    else:
        pos = torch.randperm(N, generator=g, device=DEV)[:m].sort().values.to(torch.int32)
    out = torch.empty_like(q)
    ops.attention(q, K, V, pos, out)
    mask = pos.long()[:, None] >= torch.arange(N, device=DEV)[None, :]
    ref = F.scaled_dot_product_attention(q.float().transpose(0, 1)[None], K.float()[None], V.float()[None],
                                         attn_mask=mask, enable_gqa=True)[0].transpose(0, 1)
    assert rel_err(out, ref) <= 1e-2
    assert row_rel_err(out, ref) <= 2e-2  # every (token, head) row against its own magnitude


def _attention_case(Hq, H, D, N, m, seed, sort=True):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn((m, Hq, D), generator=g, device=DEV).to(BF)
    K = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    V = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    pos = torch.randperm(N, generator=g, device=DEV)[:m]
    pos = (pos.sort().values if sort else pos).to(torch.int32)
    return q, K, V, pos


@pytest.mark.parametrize("Hq,H,D,N,m", [(28, 4, 128, 5248, 938), (28, 4, 128, 3000, 3000), (5, 1, 128, 9000, 2000)])
def test_attention_schedules_agree(Hq, H, D, N, m):
    """The persistent kernel's three schedules: slots from the workspace counter with key
    splits, the counter without splits, and static slots (no workspace).  The two
    unsplit ones compute every row the same way, bit for bit; the split one within
    bf16 rounding.  Every launch leaves the scheduler words at zero."""
    q, K, V, pos = _attention_case(Hq, H, D, N, m, seed=m)
    if m == N:
        pos = torch.arange(N, device=DEV, dtype=torch.int32)
    need = ops.attention_workspace_bytes(m, Hq, H, D, N)
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    split_out, dyn_out, static_out = (torch.empty_like(q) for _ in range(3))
    for _ in range(3):  # repeated launches reuse the same scheduler words
        ops.attention(q, K, V, pos, split_out, workspace=ws)
    ops.attention(q, K, V, pos, dyn_out, workspace=ws[:ops.ATTN_SCHED_BYTES])
    ops.attention(q, K, V, pos, static_out, workspace=ws[:0])
    torch.cuda.synchronize()
    assert int(ws[:8].count_nonzero()) == 0
    assert torch.equal(dyn_out, static_out)
    mask = pos.long()[:, None] >= torch.arange(N, device=DEV)[None, :]
    ref = F.scaled_dot_product_attention(q.float().transpose(0, 1)[None], K.float()[None], V.float()[None],
                                         attn_mask=mask, enable_gqa=True)[0].transpose(0, 1)
    assert rel_err(split_out, ref) <= 1e-2
    assert rel_err(dyn_out, ref) <= 1e-2
    assert row_rel_err(split_out, ref) <= 2e-2 and row_rel_err(dyn_out, ref) <= 2e-2


@pytest.mark.parametrize("pos", [0, 63, 64, 2000, 4099])
def test_decode_attention_matches_tensor_core_path(pos):
    """One query token: the split-KV decode kernel (workspace from attention_workspace_bytes)
    against the tensor-core kernel (no workspace) and masked SDPA, at positions on and
    next to the 64-key chunk edges."""
    Hq, H, D, N = 28, 4, 128, 4100
    g = torch.Generator(device=DEV).manual_seed(pos)
    q = torch.randn((1, Hq, D), generator=g, device=DEV).to(BF)
    K = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    V = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    p = torch.tensor([pos], dtype=torch.int32, device=DEV)
    ws = torch.zeros(ops.attention_workspace_bytes(1, Hq, H, D, N), dtype=torch.uint8, device=DEV)
    dec, tc = torch.empty_like(q), torch.empty_like(q)
    ops.attention(q, K, V, p, dec, workspace=ws)
    ops.attention(q, K, V, p, tc, workspace=ws[:0])
    mask = p.long()[:, None] >= torch.arange(N, device=DEV)[None, :]
    ref = F.scaled_dot_product_attention(q.float().transpose(0, 1)[None], K.float()[None], V.float()[None],
                                         attn_mask=mask, enable_gqa=True)[0].transpose(0, 1)
    assert rel_err(dec, ref) <= 1e-2 and rel_err(tc, ref) <= 1e-2
    assert rel_err(dec, tc) <= 1e-2


def test_attention_position_out_of_range_is_reported_not_faulted():
    """A position past the cache is clamped by the kernels and reported in the device
    error word (bit 0x8), on the split-KV decode path and on the tensor-core path."""
    Hq, H, D, N = 28, 4, 128, 300
    g = torch.Generator(device=DEV).manual_seed(5)
    q = torch.randn((1, Hq, D), generator=g, device=DEV).to(BF)
    K = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    V = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    p = torch.tensor([N + 5], dtype=torch.int32, device=DEV)
    ws = torch.zeros(ops.attention_workspace_bytes(1, Hq, H, D, N), dtype=torch.uint8, device=DEV)
    out = torch.empty_like(q)
    ops.attention(q, K, V, p, out, workspace=ws)
    assert _lib.device_error() & 0x8
    ops.attention(q, K, V, p, out, workspace=ws[:0])
    assert _lib.device_error() & 0x8
    assert torch.isfinite(out.float()).all()


def test_attention_unsorted_positions():
    """Row blocks whose positions are not sorted: each row still sees exactly its keys."""
    Hq, H, D, N, m = 28, 4, 128, 2600, 500
    q, K, V, pos = _attention_case(Hq, H, D, N, m, seed=7, sort=False)
    out = torch.empty_like(q)
    ops.attention(q, K, V, pos, out)
    mask = pos.long()[:, None] >= torch.arange(N, device=DEV)[None, :]
    ref = F.scaled_dot_product_attention(q.float().transpose(0, 1)[None], K.float()[None], V.float()[None],
                                         attn_mask=mask, enable_gqa=True)[0].transpose(0, 1)
    assert rel_err(out, ref) <= 1e-2


# ------------------------------------------------------------- elementwise
@pytest.mark.parametrize("hid", [64, 896, 3584, 5120])
def test_rmsnorm_matches_reference_formula(hid):
    x = torch.randn((77, hid), device=DEV).to(BF)
    w = (1 + 0.1 * torch.randn(hid, device=DEV)).to(BF)
    y = ops.rmsnorm(x, w, 1e-6)
    x32 = x.float()
    ref = w * (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + 1e-6)).to(BF)
    assert rel_err(y, ref) <= 1e-2
    assert (y != ref).float().mean() < 0.01


@pytest.mark.parametrize("hid", [896, 5120])
def test_add_rmsnorm_is_residual_add_then_rmsnorm(hid):
    h = torch.randn((53, hid), device=DEV).to(BF)
    dlt = torch.randn((53, hid), device=DEV).to(BF)
    w = (1 + 0.1 * torch.randn(hid, device=DEV)).to(BF)
    h_ref = h + dlt  # bf16 add: fp32 sum rounded once
    x = torch.empty_like(h)
    ops.add_rmsnorm(h, dlt, w, 1e-6, x)
    assert torch.equal(h, h_ref)
    assert torch.equal(x, ops.rmsnorm(h_ref, w, 1e-6))


def test_rmsnorm_embed_gemv_log_softmax():
    hid, vocab = 896, 5000
    x = torch.randn((77, hid), device=DEV).to(BF)
    E = torch.randn((vocab, hid), device=DEV).to(BF)
    toks = torch.randint(0, vocab, (200,), device=DEV, dtype=torch.int32)
    rows = torch.randperm(200, device=DEV)[:50].sort().values.to(torch.int32)
    out = torch.empty((50, hid), dtype=BF, device=DEV)
    ops.embed(E, toks, rows, out)
    assert torch.equal(out, E[toks[rows.long()].long()])
    for mm in (1, 3, 8):
        xx = x[:mm].contiguous()
        lo = ops.gemv(xx, E)
        assert rel_err(lo, xx.float() @ E.float().T) <= 1e-2
    # the row is split over an 8-CTA cluster: sizes with empty and ragged slices, the 7B vocab
    for n in (vocab, 1, 5, 9, 8191, 152064):
        row = (torch.randn(n, device=DEV) * 5).to(BF)
        lp = ops.log_softmax(row)
        torch.testing.assert_close(lp, torch.log_softmax(row.float(), -1), rtol=1e-5, atol=1e-5)
        assert torch.equal(lp, ops.log_softmax(row)), "the cluster's combine must be deterministic"


def test_greedy_next_is_torch_argmax_and_advances_the_position():
    g = torch.Generator(device=DEV).manual_seed(7)
    tok = torch.zeros(1, dtype=torch.int32, device=DEV)
    pos = torch.full((1,), 41, dtype=torch.int32, device=DEV)
    rows = [(torch.randn(n, generator=g, device=DEV) * 4).to(BF) for n in (1, 5, 9, 5000, 152064)]
    tied = torch.randint(0, 3, (152064,), generator=g, device=DEV).to(BF)  # the max repeats ~50k times
    rows.append(tied)
    late = torch.full((152064,), -3.0, device=DEV).to(BF)
    late[-1] = 2.0  # the winner in the last slice
    rows.append(late)
    nan = rows[3].clone()
    nan[[17, 4000]] = float("nan")  # torch.argmax returns the first NaN
    rows.append(nan)
    for i, row in enumerate(rows):
        ops.greedy_next(row, tok, pos)
        assert int(tok) == int(torch.argmax(row)), i
        assert int(pos) == 42 + i
    ops.greedy_next(rows[0], tok)  # no position: only the token is written
    assert int(tok) == 0 and int(pos) == 41 + len(rows)
