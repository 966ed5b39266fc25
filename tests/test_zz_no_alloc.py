"""The allocation-free selection entry point, called through the C ABI.

ckv_deviation_select_noalloc exists for callers that own their inputs and outputs
but cannot allocate the two scratch buffers ckv_deviation_select asks for (a
serving loop whose device memory belongs to its own arena, or a C/FFI host with
no allocator at hand); its scratch is a static device array inside the library.
Here it must give the same results as ckv_deviation_select with caller-provided
scratch, on two calls in a row (the shared scratch is reused between calls).
This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from chunkkv_b200 import _lib, ops  # noqa: E402

DEV = "cuda"
BF = torch.bfloat16
NOALLOC_MAX_CTX = 65536  # CKV_NOALLOC_MAX_CTX in include/chunkkv_b200.h


def _inputs(seed=7):
    H, D, n_ch, cl = 4, 128, 8, 256
    N = n_ch * cl + 96  # cached chunks, then fresh query tokens
    g = torch.Generator(device=DEV).manual_seed(seed)
    Kb = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    Vb = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    kf = Kb.permute(1, 0, 2).reshape(N, H * D).clone()
    vf = Vb.permute(1, 0, 2).reshape(N, H * D).clone()
    noisy = torch.rand(N, generator=g, device=DEV) < 0.2
    kf[noisy] = (kf[noisy].float() + 0.05 * torch.randn(kf[noisy].shape, generator=g, device=DEV)).to(BF)
    vf[noisy] = (vf[noisy].float() + 0.05 * torch.randn(vf[noisy].shape, generator=g, device=DEV)).to(BF)
    flags = torch.zeros(N, dtype=torch.uint8)
    flags[:n_ch * cl] = 1
    for c in range(n_ch):
        flags[c * cl:c * cl + 4] |= 2
    meta = torch.tensor([[c * cl, cl, 38, 0] for c in range(n_ch)], dtype=torch.int32, device=DEV)
    active = torch.arange(N, dtype=torch.int32, device=DEV)
    return dict(kf=kf, vf=vf, Kb=Kb, Vb=Vb, active=active, flags=flags.to(DEV), meta=meta, N=N, H=H, D=D)


def _outputs(N, n_ch):
    f32 = dict(dtype=torch.float32, device=DEV)
    i32 = dict(dtype=torch.int32, device=DEV)
    return dict(diff=torch.full((N,), -1.0, **f32), norm=torch.full((N,), -1.0, **f32),
                rel=torch.zeros(n_ch, **f32), keep_abs=torch.full((N,), -1, **i32),
                sel=torch.full((N,), -1, **i32), counts=torch.full((8,), -1, **i32))


def _noalloc(x, o, thr=None):
    s = torch.cuda.current_stream().cuda_stream
    p = lambda t: t.data_ptr()  # noqa: E731
    _lib.call("ckv_deviation_select_noalloc", p(x["kf"]), p(x["vf"]), x["kf"].stride(0), p(x["Kb"]),
              p(x["Vb"]), p(x["active"]), x["active"].numel(), p(x["flags"]), x["N"], p(x["meta"]), x["meta"].shape[0],
              int(thr is not None), float(thr or 0.0), x["H"], x["D"], p(o["diff"]), p(o["norm"]),
              p(o["rel"]), p(o["keep_abs"]), p(o["sel"]), p(o["counts"]), s)


def test_noalloc_matches_caller_scratch_entry_point_twice():
    x = _inputs()
    n_ch = x["meta"].shape[0]
    ws = ops.SelectWorkspace(x["N"], n_ch, DEV)
    ops.deviation_select(x["kf"], x["vf"], x["Kb"], x["Vb"], x["active"], x["flags"], x["meta"], None, ws)
    torch.cuda.synchronize()
    n_ref = int(ws.counts[0])
    assert n_ref == 8 * 38 + 8 * 4 + 96
    for _ in range(2):  # two calls in a row share (and must reset) the built-in scratch
        o = _outputs(x["N"], n_ch)
        _noalloc(x, o)
        torch.cuda.synchronize()
        torch.testing.assert_close(o["diff"], ws.diff[:x["N"]], rtol=1e-4, atol=1e-6)
        torch.testing.assert_close(o["norm"], ws.norm[:x["N"]], rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(o["rel"], ws.rel[:n_ch], rtol=1e-4, atol=0)
        assert torch.equal(o["counts"], ws.counts)
        np.testing.assert_array_equal(o["keep_abs"][:n_ref].cpu().numpy(), ws.keep_abs[:n_ref].cpu().numpy())
        np.testing.assert_array_equal(o["sel"][:n_ref].cpu().numpy(), ws.sel[:n_ref].cpu().numpy())
    assert _lib.device_error() == 0


def _boundary_inputs(seed=11):
    """n_ctx = CKV_NOALLOC_MAX_CTX: one long exact chunk (never computed, not active),
    then four moved chunks and a query; only those 592 positions are active.  At this
    size the selection keeps its per-position keys in the built-in array, up to its
    last byte."""
    H, D, N = 4, 128, NOALLOC_MAX_CTX
    n_ch, cl, q = 4, 128, 80
    tail0 = N - n_ch * cl - q
    g = torch.Generator(device=DEV).manual_seed(seed)
    Kb = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    Vb = torch.randn((H, N, D), generator=g, device=DEV).to(BF)
    active = torch.arange(tail0, N, dtype=torch.int32, device=DEV)
    n_act = active.numel()
    kf = Kb[:, tail0:].permute(1, 0, 2).reshape(n_act, H * D).clone()
    vf = Vb[:, tail0:].permute(1, 0, 2).reshape(n_act, H * D).clone()
    kf += (0.05 * torch.randn(kf.shape, generator=g, device=DEV)).to(BF)
    vf[: n_act // 2] += (0.2 * torch.randn((n_act // 2, H * D), generator=g, device=DEV)).to(BF)
    flags = torch.zeros(N, dtype=torch.uint8)
    flags[:tail0] = 1 | 4  # cached, exact
    meta = [[0, tail0, -1, 1]]
    for c in range(n_ch):
        s0 = tail0 + c * cl
        flags[s0:s0 + cl] = 1
        flags[s0:s0 + 4] |= 2
        meta.append([s0, cl, 19, 0])
    return dict(kf=kf, vf=vf, Kb=Kb, Vb=Vb, active=active, flags=flags.to(DEV),
                meta=torch.tensor(meta, dtype=torch.int32, device=DEV), N=N, H=H, D=D, n_act=n_act)


def _compare(x, thr):
    """Workspace entry point vs the built-in-scratch entry point, two calls in a row."""
    n_ch = x["meta"].shape[0]
    ws = ops.SelectWorkspace(x["N"], n_ch, DEV)
    ops.deviation_select(x["kf"], x["vf"], x["Kb"], x["Vb"], x["active"], x["flags"], x["meta"], thr, ws)
    torch.cuda.synchronize()
    n_ref = int(ws.counts[0])
    act = x["active"].long()
    for _ in range(2):
        o = _outputs(x["N"], n_ch)
        _noalloc(x, o, thr)
        torch.cuda.synchronize()
        torch.testing.assert_close(o["diff"][act], ws.diff[act], rtol=1e-4, atol=1e-6)
        torch.testing.assert_close(o["rel"], ws.rel[:n_ch], rtol=1e-4, atol=0, equal_nan=True)
        assert torch.equal(o["counts"], ws.counts)
        np.testing.assert_array_equal(o["keep_abs"][:n_ref].cpu().numpy(), ws.keep_abs[:n_ref].cpu().numpy())
        np.testing.assert_array_equal(o["sel"][:n_ref].cpu().numpy(), ws.sel[:n_ref].cpu().numpy())
    assert _lib.device_error() == 0
    return ws


def test_noalloc_at_its_maximum_size():
    x = _boundary_inputs()
    ws = _compare(x, None)
    n = int(ws.counts[0])
    assert n == 4 * 19 + 4 * 4 + 80 and int(ws.counts[2]) == 76
    assert int(ws.keep_abs[0]) >= NOALLOC_MAX_CTX - 4 * 128 - 80 and int(ws.keep_abs[n - 1]) == NOALLOC_MAX_CTX - 1


def test_noalloc_with_escalation_threshold():
    x = _inputs(seed=9)
    # the first two chunks deviate strongly: a threshold between them and the rest
    # escalates exactly those two (their whole spans are kept)
    for c in (0, 1):
        sl = slice(c * 256, (c + 1) * 256)
        x["kf"][sl] = (x["kf"][sl].float() * 1.5).to(BF)
    ws = _compare(x, 0.05)
    assert int(ws.counts[4]) == 0b11
    kept = ws.keep_abs[:int(ws.counts[0])].cpu().numpy()
    assert np.isin(np.arange(512), kept).all()
    # at the maximum size: chunks 1 and 2 of the table (the first 256 moved positions)
    # carry the larger V noise, relative deviation about 0.02 against about 0.001
    x2 = _boundary_inputs(seed=12)
    ws2 = _compare(x2, 0.01)
    assert int(ws2.counts[4]) == 0b110


def test_noalloc_rejects_sizes_beyond_its_scratch():
    x = _inputs()
    o = _outputs(x["N"], x["meta"].shape[0])
    x = dict(x, N=NOALLOC_MAX_CTX + 1)
    with pytest.raises(ValueError, match="scratch"):
        _noalloc(x, o)
