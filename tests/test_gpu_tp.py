"""Tensor-parallel blend prefill on 2 GPUs, against the reference fixtures and against the
same engine on one GPU, with both exchanges: partial rows read over NVLink peer memory by
the owning ranks (`ckv_linear_partial` + `ckv_reduce_add_gather`, the default) and the NCCL
all-reduce.

Each rank holds one of the two KV heads of the `tiny` shape with its query heads
and half of the MLP.  Checked per scenario, on every rank:
  - stats (token counts, recomputed count, prefill_token_equiv, escalations) equal
    the reference fixture's, and the first-token logit KL against it is <= 1e-3;
  - selection bit-exact given the scores: the all-reduced layer-1 scores fed to the
    oracle's selection give exactly the kept positions of the engine;
  - every rank ends with the same selection and bit-identical logits (replicated
    state stays in step);
  - rank r's blended K/V equal head r of a one-GPU run within bf16 tolerance.
Needs 2 GPUs; skipped otherwise.  NVLS is off (NCCL_NVLS_ENABLE=0).
"""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
TINY = ["tiny_fp32", "tiny_bf16", "tiny_escalate", "tiny_exact_overflow"]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        from chunkkv_b200 import _lib
        from chunkkv_b200.engine.tp import TensorParallel
        from chunkkv_b200.engine.torch_engine import TorchEngine
        from chunkkv_b200.engine.weights import pack
        from helpers import kl, run_blend, scenario
        from oracle.blend_oracle import select

        out = {}
        for fused in (True, False):
            tp = TensorParallel(fused=fused)
            for name in TINY:
                s = scenario(name)
                eng = TorchEngine.from_packed(pack(s.shape, s.sd, device=dev, tp_rank=rank, tp_size=world), tp=tp)
                _, _, pl, res = run_blend(eng, s)
                torch.cuda.synchronize()
                N = len(s.tokens)
                cached = torch.zeros(N, dtype=torch.bool)
                sink = torch.zeros(N, dtype=torch.bool)
                for p in pl:
                    cached[p.start:p.start + p.chunk.length] = True
                    if not p.exact:
                        sink[p.start:min(p.start + p.chunk.length, p.start + s.config.n_sink)] = True
                ws = eng._ws
                sel = res.selected.cpu().numpy()
                ref_sel = select(ws.diff[:N].cpu(), ws.norm[:N].cpu(), cached, sink, pl, s.config)["keep_abs"].numpy()
                single = TorchEngine.from_packed(pack(s.shape, s.sd, device=dev))
                _, _, _, res1 = run_blend(single, s)
                K1, V1 = res1.cache
                K2, V2 = res.cache
                hs = slice(rank * K2.shape[1], (rank + 1) * K2.shape[1])

                def rel(a, b):
                    a, b = a.float(), b.float()
                    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))

                # positions both runs recomputed or both moved (near-tied selections may differ)
                same = np.ones(N, bool)
                diff_sel = np.setxor1d(sel, res1.selected.cpu().numpy())
                same[diff_sel] = False
                same_t = torch.from_numpy(same).to(dev)
                out[(name, fused)] = {
                    "stats": {k: res.stats[k] for k in ("tokens", "cached_tokens", "recomputed_cached_tokens",
                                                        "prefill_token_equiv")},
                    "escalated": [c["escalated"] for c in res.stats["chunks"]],
                    "kl_ref": kl(s.arrays["logits"][-1].astype(np.float32), res.logits[-1].float().cpu().numpy()),
                    "kl_single": kl(res1.logits[-1].float().cpu().numpy(), res.logits[-1].float().cpu().numpy()),
                    "sel_exact": bool(np.array_equal(ref_sel, sel)),
                    "selected": sel.tolist(),
                    "logits": res.logits[-1].float().cpu().numpy(),
                    "kv_rel": max(rel(K2[:, :, same_t], K1[:, hs][:, :, same_t]),
                                  rel(V2[:, :, same_t], V1[:, hs][:, :, same_t])),
                }
                del eng, single
            if tp._exchange is not None:
                tp._exchange.close()
        _lib.check_device()
        q.put((rank, out))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_2gpu_matches_reference_and_single_gpu(golden):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, o = q.get(timeout=600)
        res[r] = o
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in (0, 1):
        assert isinstance(res[r], dict), res[r]
    for name, fused in [(n, f) for n in TINY for f in (True, False)]:
        meta, _ = golden(name)
        for r in (0, 1):
            o = res[r][(name, fused)]
            for k, v in o["stats"].items():
                assert v == meta["stats"][k], (name, r, k)
            assert o["escalated"] == [c["escalated"] for c in meta["stats"]["chunks"]], (name, r)
            assert o["kl_ref"] <= 1e-3 and o["kl_single"] <= 1e-3, (name, r, o["kl_ref"], o["kl_single"])
            assert o["sel_exact"], (name, r)
            assert o["kv_rel"] <= 1e-2, (name, r, o["kv_rel"])
        assert res[0][(name, fused)]["selected"] == res[1][(name, fused)]["selected"], name
        assert np.array_equal(res[0][(name, fused)]["logits"], res[1][(name, fused)]["logits"]), name


def _worker_32b(rank, world, port, q):
    """Truncated 32B shape (3 layers, hidden 5120, 40 Q / 8 KV heads = 5:1 GQA, head_dim
    128, intermediate 27648), 8 x 256 shuffled chunks + 64-token query, 15 % + 4 sinks,
    split by KV head over `world` ranks, against the bf16 oracle on the same cached
    chunks (the first prefill's K/V, gathered from the ranks)."""
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import random

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        from chunkkv_b200 import _lib
        from chunkkv_b200.engine.base import BlendConfig, ChunkKV, Placement, plan_arrays
        from chunkkv_b200.engine.tp import TensorParallel
        from chunkkv_b200.engine.torch_engine import TorchEngine
        from chunkkv_b200.engine.weights import SHAPES, pack, random_state_dict
        from helpers import kl
        from oracle.blend_oracle import OracleEngine, select

        shape = SHAPES["qwen2.5-32b"].truncated(3)
        sd = random_state_dict(shape, seed=0, dtype=torch.bfloat16, device=dev)  # same values on every rank
        w_local = pack(shape, sd, device=dev, tp_rank=rank, tp_size=world)
        sd_cpu = {k: v.cpu() for k, v in sd.items()}
        del sd
        torch.cuda.empty_cache()
        orc = OracleEngine(shape, sd_cpu, dtype=torch.bfloat16)
        rng = random.Random(5)
        n_ch, cl, nq = 8, 256, 64
        chunks = [[rng.randrange(shape.vocab) for _ in range(cl)] for _ in range(n_ch)]
        query = [rng.randrange(shape.vocab) for _ in range(nq)]
        order = list(range(n_ch))
        rng.shuffle(order)
        cfg = BlendConfig(recompute_ratio=0.15, n_sink=4)
        out = {}
        for fused in (True, False):
            tp = TensorParallel(fused=fused)
            eng = TorchEngine.from_packed(w_local, tp=tp)
            first = eng.prefill(sum(chunks, []))
            K, V = first.cache  # this rank's heads [L, H/world, n, D]
            Kf = [torch.empty_like(K) for _ in range(world)]
            Vf = [torch.empty_like(V) for _ in range(world)]
            dist.all_gather(Kf, K.contiguous())
            dist.all_gather(Vf, V.contiguous())
            Kall, Vall = torch.cat(Kf, 1).cpu(), torch.cat(Vf, 1).cpu()  # all heads, in rank order
            local = [first.chunk(i * cl, (i + 1) * cl) for i in range(n_ch)]
            tokens, pl, pl_cpu = [], [], []
            for c in order:
                pl.append(Placement(local[c], len(tokens)))
                sl = slice(c * cl, (c + 1) * cl)
                pl_cpu.append(Placement(ChunkKV([Kall[li, None, :, sl].contiguous() for li in range(shape.n_layers)],
                                                [Vall[li, None, :, sl].contiguous() for li in range(shape.n_layers)],
                                                c * cl), len(tokens)))
                tokens += chunks[c]
            tokens += query
            N = len(tokens)
            res = eng.prefill(tokens, pl, cfg)
            torch.cuda.synchronize()
            ores = orc.prefill(tokens, pl_cpu, cfg)
            plan = plan_arrays(N, pl, cfg.n_sink)
            ws = eng._ws
            sel = res.selected.cpu().numpy()
            mine = select(ws.diff[:N].cpu(), ws.norm[:N].cpu(), torch.from_numpy(plan.cached),
                          torch.from_numpy(plan.sink), pl, cfg)["keep_abs"].numpy()
            o_sel = ores.keep_abs.numpy()
            moved = np.ones(N, bool)
            moved[sel] = False
            moved[o_sel] = False
            moved[~plan.cached] = False
            mv = torch.from_numpy(moved)
            Kr, Vr = res.cache
            hl = Kr.shape[1]
            hs = slice(rank * hl, (rank + 1) * hl)

            def rel(a, b):
                a, b = a.float().cpu(), b.float().cpu()
                return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))

            kv = max(max(rel(Kr[li][:, mv.to(dev)], ores.keys[li][0][hs][:, mv]),
                          rel(Vr[li][:, mv.to(dev)], ores.values[li][0][hs][:, mv])) for li in range(shape.n_layers))
            out[fused] = {"sel_exact": bool(np.array_equal(mine, sel)), "kv_rel": kv,
                          "kl": kl(ores.logits[-1].float().numpy(), res.logits[-1].float().cpu().numpy()),
                          "jaccard": len(np.intersect1d(sel, o_sel)) / len(np.union1d(sel, o_sel)),
                          "budget": (int(sum(int(round(0.15 * cl)) for _ in pl)), ores.budget),
                          "n_sel": len(sel), "selected": sel.tolist()}
            del eng, first, res
            if tp._exchange is not None:
                tp._exchange.close()
        _lib.check_device()
        q.put((rank, out))
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_2gpu_truncated_32b_matches_oracle():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_32b, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, o = q.get(timeout=900)
        res[r] = o
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in (0, 1):
        assert isinstance(res[r], dict), res[r]
        for fused in (True, False):
            o = res[r][fused]
            assert o["sel_exact"], (r, fused)
            assert o["kv_rel"] <= 1e-2, (r, fused, o["kv_rel"])
            assert o["kl"] <= 1e-3, (r, fused, o["kl"])
            assert o["jaccard"] >= 0.85, (r, fused, o["jaccard"])
            assert o["budget"][0] == o["budget"][1]
            assert o["n_sel"] == o["budget"][0] + 8 * 4 + 64
    for fused in (True, False):
        assert res[0][fused]["selected"] == res[1][fused]["selected"]


def test_exchange_wait_runs_out_and_reports_without_a_peer():
    """Failure detection on one GPU: the reduce kernel of a 2-rank exchange whose peer
    never signals gives up after its bounded wait (2 s), records CKV_DEV_ERR_WAIT_TIMEOUT
    and returns; the host reads the error word and the GPU stays usable."""
    from chunkkv_b200 import _lib, ops

    dev = torch.device("cuda", 0)
    rows, hidden = 64, 256
    bf = torch.bfloat16
    parts = [torch.zeros((rows, hidden), dtype=bf, device=dev) for _ in range(2)]
    hs = [torch.zeros((rows, hidden), dtype=bf, device=dev) for _ in range(2)]
    ctl = torch.zeros(64, dtype=torch.int32, device=dev)  # counters: nothing ever signals them

    def table(ts):
        return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64).view(torch.uint64).to(dev)

    part_tab, h_tab = table(parts), table(hs)
    gather_tab = table([ctl[8:], ctl[8:]])
    _lib.check_device()  # start from a clean error word
    _lib.call("ckv_reduce_add_gather", part_tab.data_ptr(), 0, 2, rows, hidden, hs[0].data_ptr(),
              h_tab.data_ptr(), ctl.data_ptr(), ctl[8:].data_ptr(), gather_tab.data_ptr(),
              ctl[16:].data_ptr(), 1, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _lib.device_error() & 0x1  # CKV_DEV_ERR_WAIT_TIMEOUT
    # the context is intact: an ordinary kernel still runs and the error word is clear
    x = torch.randn((8, hidden), device=dev).to(bf)
    y = ops.rmsnorm(x, torch.ones(hidden, dtype=bf, device=dev), 1e-6)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    _lib.check_device()
