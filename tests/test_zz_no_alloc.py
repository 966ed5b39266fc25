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
              p(x["Vb"]), p(x["active"]), x["N"], p(x["flags"]), x["N"], p(x["meta"]), x["meta"].shape[0],
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


def test_noalloc_rejects_sizes_beyond_its_scratch():
    x = _inputs()
    o = _outputs(x["N"], x["meta"].shape[0])
    x = dict(x, N=NOALLOC_MAX_CTX + 1)
    with pytest.raises(ValueError, match="scratch"):
        _noalloc(x, o)
