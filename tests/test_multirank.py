"""Multi-rank host logic on 2 CPU ranks (gloo): the bench's max-over-ranks timing
reduction, per-rank request streams, a peer that dies before a collective (the
survivor gets an error from the short process-group timeout, no hang), and the
tensor-parallel weight shards: each rank's column-parallel outputs are its slice of
the full layer's, and the sum over ranks of the row-parallel partials (o_proj,
down_proj) and of the per-head deviation scores is the full layer's result."""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        if mode == "tp_shards":
            q.put((rank, _tp_shard_check(rank, world)))
        elif mode == "max":
            q.put((rank, bench.max_over_ranks(1.5 + rank), bench.request_seed(rank)))
        elif mode == "peer_dies":
            if rank == 1:
                os._exit(0)  # leaves between steps, no collective in flight
            try:
                bench.max_over_ranks(1.0)
                q.put((rank, "no error"))
            except Exception as e:  # noqa: BLE001
                q.put((rank, f"error: {type(e).__name__}"))
    finally:
        if mode != "peer_dies":
            dist.destroy_process_group()


def _tp_shard_check(rank, world):
    """Errors (max abs) of the sharded layer against the unsharded one, in fp32."""
    import torch
    import torch.nn.functional as F

    from chunkkv_b200.engine.tp import TensorParallel
    from chunkkv_b200.engine.weights import GU_BLOCK, SHAPES, pack, random_state_dict

    tp = TensorParallel()
    shape = SHAPES["tiny"]
    sd = random_state_dict(shape, seed=0, dtype=torch.float32)
    full = pack(shape, sd, device="cpu")
    mine = pack(shape, sd, device="cpu", tp_rank=rank, tp_size=world)
    loc = mine.shape
    assert (mine.tp_rank, mine.tp_size) == (rank, world)
    assert (loc.n_heads, loc.n_kv, loc.inter) == (shape.n_heads // world, shape.n_kv // world,
                                                  shape.inter // world)
    D, M, hid = shape.head_dim, 37, shape.hidden
    g = torch.Generator().manual_seed(5)
    x = torch.randn(M, hid, generator=g)
    attn = torch.randn(M, shape.n_heads * D, generator=g)
    fresh_k = torch.randn(M, shape.n_kv * D, generator=g)
    base_k = torch.randn(M, shape.n_kv * D, generator=g)
    err = {}
    lf, lm = full.layers[1], mine.layers[1]
    # column-parallel QKV: this rank's q, k, v columns
    qkv_f = x @ lf.w_qkv.float().T + lf.b_qkv.float()
    qkv_m = x @ lm.w_qkv.float().T + lm.b_qkv.float()
    Hq, H, hq, hk = shape.n_heads, shape.n_kv, loc.n_heads, loc.n_kv
    q_f = qkv_f[:, :Hq * D][:, rank * hq * D:(rank + 1) * hq * D]
    k_f = qkv_f[:, Hq * D:(Hq + H) * D][:, rank * hk * D:(rank + 1) * hk * D]
    v_f = qkv_f[:, (Hq + H) * D:][:, rank * hk * D:(rank + 1) * hk * D]
    err["qkv"] = (torch.cat([q_f, k_f, v_f], 1) - qkv_m).abs().max().item()
    # row-parallel o_proj: partial of this rank's heads, summed over ranks
    part = attn[:, rank * hq * D:(rank + 1) * hq * D] @ lm.w_o.float().T
    tp.all_reduce_(part)
    err["o_proj"] = (part - attn @ lf.w_o.float().T).abs().max().item()

    # gate/up (interleaved 128-row blocks) column-parallel, down row-parallel
    def mlp(w_gu, w_down):
        blocks = w_gu.float().view(-1, 2, GU_BLOCK, hid)
        gate, up = blocks[:, 0].reshape(-1, hid), blocks[:, 1].reshape(-1, hid)
        return (F.silu(x @ gate.T) * (x @ up.T)) @ w_down.float().T

    part = mlp(lm.w_gu, lm.w_down)
    tp.all_reduce_(part)
    err["mlp"] = (part - mlp(lf.w_gu, lf.w_down)).abs().max().item()
    # deviation scores: per-head partial sums add up to the all-head sum
    sl = slice(rank * hk * D, (rank + 1) * hk * D)
    d = ((fresh_k[:, sl] - base_k[:, sl]) ** 2).sum(1)
    tp.all_reduce_(d)
    err["scores"] = (d - ((fresh_k - base_k) ** 2).sum(1)).abs().max().item()
    err["replicated"] = float(not (torch.equal(mine.embed, full.embed) and torch.equal(mine.norm, full.norm)
                                   and torch.equal(lm.ln1, lf.ln1) and torch.equal(lm.ln2, lf.ln2)))
    return err


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    out = []
    while not q.empty():
        out.append(q.get())
    for p in procs:
        if p.is_alive():
            p.kill()
    return out


def test_max_over_ranks_and_distinct_request_streams():
    out = sorted(_run("max"))
    assert [o[1] for o in out] == [2.5, 2.5]
    assert out[0][2] != out[1][2]


def test_dead_peer_gives_an_error_not_a_hang():
    out = _run("peer_dies")
    assert out and out[0][0] == 0 and out[0][1].startswith("error"), out


def test_tensor_parallel_shards_reassemble_the_layer():
    out = dict(_run("tp_shards"))
    assert sorted(out) == [0, 1], out
    for rank, err in out.items():
        assert err["qkv"] < 1e-5 and err["replicated"] == 0.0, (rank, err)
        assert err["o_proj"] < 1e-4 and err["mlp"] < 1e-4 and err["scores"] < 1e-3, (rank, err)


def test_tp_local_refuses_uneven_splits():
    import pytest

    from chunkkv_b200.engine.weights import SHAPES

    s = SHAPES["qwen2.5-32b"]
    assert s.tp_local(8).n_kv == 1 and s.tp_local(8).inter == 3456 and s.tp_local(8).n_heads == 5
    with pytest.raises(NotImplementedError):
        SHAPES["qwen2.5-7b"].tp_local(8)  # 4 KV heads
    with pytest.raises(NotImplementedError):
        SHAPES["tiny7"].tp_local(2)  # 1 KV head
