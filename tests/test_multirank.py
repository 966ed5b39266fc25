"""Data-parallel host logic on 2 CPU ranks (gloo): the bench's max-over-ranks timing
reduction, per-rank request streams, and a peer that dies before a collective
(the survivor gets an error from the short process-group timeout, no hang)."""

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
        if mode == "max":
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
