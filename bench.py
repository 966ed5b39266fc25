#!/usr/bin/env python
"""Blend-prefill benchmark (Qwen2.5-7B shape on one B200).

Workload per step: one blend prefill of a request made of 10 cached chunks x 512
tokens served in a seeded random permutation plus a 128-token query (N = 5248),
15 % recompute + 4 sink tokens per chunk, through TorchEngine.prefill.  Weights
are random-init bf16 (seed 0); chunk K/V come from a full prefill of the chunks
in their original order, stored in the paged HBM store (untimed setup).

    python bench.py [--gpus N --steps K --warmup W]            # this engine
    python bench.py --impl reference [...]                      # CPU reference arm

Under torchrun each rank serves its own request stream on its own GPU (data
parallel by request, no collective on the data path); times are the max over
ranks.  One JSON line is printed by rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# Per-kernel times (the `kernels` table and the roofline): a second pass of the same steps
# with a CUDA-event pair around every launch, each pair preceded by a device sleep so that
# the launch is already queued when its start event runs.
KERNEL_GATE_US = 50.0
KERNEL_TIMING = (f"CUDA-event pair around each launch in a second pass of the same steps; a "
                 f"{KERNEL_GATE_US:.0f} us device sleep before each pair keeps the host's submission "
                 f"time out of it (no dependent-launch overlap inside a pair)")
METRIC = "blend-prefill tokens/s (Qwen2.5-7B shape, 10x512 shuffled cached chunks + 128-token query)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ratio", type=float, default=0.15)
    ap.add_argument("--n-sink", type=int, default=4)
    ap.add_argument("--workload", choices=["dp", "tp", "replay", "micro", "decode", "policies"], default="dp",
                    help="dp: config 3 (7B, one request per GPU); tp: config 5 (32B split over the GPUs "
                         "by KV head, 64x512 chunks; defaults --shape qwen2.5-32b --chunks 64 --steps 10); "
                         "replay: config 4 (256 requests over a 16x256 chunk pool, split over the GPUs); "
                         "micro: config 2 (the K/V bandwidth kernels at the 7B KV shape, one GPU); "
                         "decode: greedy decode after the config-3 blend prefill (one GPU); "
                         "policies: a synthetic multi-tenant stream under P0-P4 with TTFT, compute, KL and "
                         "greedy agreement against P0 (one GPU)")
    ap.add_argument("--requests", type=int, default=256,
                    help="replay: total requests over all GPUs; policies: requests per policy (default 48)")
    ap.add_argument("--max-new", type=int, default=8, help="policies: greedy tokens per request")
    ap.add_argument("--tp-exchange", choices=["peer", "nccl"], default="peer",
                    help="tp: partial rows over NVLink peer memory (fused kernels) or NCCL all-reduce")
    ap.add_argument("--shape", default=None)
    ap.add_argument("--chunks", type=int, default=None)
    ap.add_argument("--chunk-len", type=int, default=512)
    ap.add_argument("--query-len", type=int, default=128)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--extra-ratios", default="0.30,0.50", help="also time these ratios (TTFT only)")
    ap.add_argument("--kernel-case", choices=["swiglu", "oproj", "down", "qkv", "attention", "gather", "deviation",
                                              "deviation_scores", "select", "decode_swiglu", "decode_down"],
                    help="time one kernel at its 7B-bench shape (for ncu captures) instead of the prefill")
    args = ap.parse_args()
    tp = args.workload == "tp"
    if args.shape is None:
        args.shape = "qwen2.5-32b" if tp else "qwen2.5-7b"
    if args.chunks is None:
        args.chunks = 64 if tp else 10
    if tp and "--steps" not in sys.argv:
        args.steps = 10
    if args.workload == "policies" and "--requests" not in sys.argv:
        args.requests = 48
    if args.workload == "replay":
        if "--ratio" not in sys.argv:
            args.ratio = 0.30
        if "--n-sink" not in sys.argv:
            args.n_sink = 2  # ChunkReuseRuntime's BlendConfig default (base.py:39)
    return args


def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            out = {k: float(d[k]) for k in FALLBACK_PEAKS}
            clk = d.get("clocks_under_load") or {}
            if isinstance(clk, dict) and clk.get("sm_mhz_median"):
                out["sustained_sm_mhz"] = float(clk["sm_mhz_median"])  # SM clock of the sustained run
            return out, "measured"
        except (OSError, ValueError, KeyError, TypeError):  # unreadable or partial: use the fallback
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def make_request(vocab: int, n_chunks: int, chunk_len: int, query_len: int, seed: int):
    rng = random.Random(seed)
    chunks = [[rng.randrange(vocab) for _ in range(chunk_len)] for _ in range(n_chunks)]
    query = [rng.randrange(vocab) for _ in range(query_len)]
    order = list(range(n_chunks))
    while order == sorted(order):
        rng.shuffle(order)
    return chunks, order, query


def max_over_ranks(x: float, device="cpu") -> float:
    """Timing reduction of the data-parallel run: the slowest rank's time (no data exchange)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def nccl_init_logging() -> None:
    """NCCL's communicator set-up lines (rank, nRanks, transports) in the output: INFO
    level for the INIT subsystem only, so the rest of the run stays quiet."""
    os.environ["NCCL_DEBUG"] = "INFO"
    os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"


def physical_index(local: int) -> int:
    """nvidia-smi index of this rank's GPU (CUDA_VISIBLE_DEVICES may renumber them)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    parts = vis.split(",") if vis else []
    return int(parts[local]) if local < len(parts) and parts[local].strip().isdigit() else local


def request_seed(rank: int) -> int:
    """Each rank serves its own request stream (data parallel by request)."""
    return 1000 + rank


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except OSError:  # no nvidia-smi: the line then reports no clock samples
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), float(f[3]), f[5:9]))
            except ValueError:
                continue
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for _, _, _, r in rows for n, v in zip(names, r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


# -------------------------------------------------------------- CPU sample
class CpuSample:
    """The reference algorithm (oracle port of torch_engine.py:80-178) on the host cores,
    on the bench's own request: every layer of the model, seed-0 random weights, the
    chunks' cached K/V at N(0, 1) scale.  It computes in the dtype the host multiplies
    fastest, bf16 (the reference's deployment dtype) when the host has native bf16
    matrix units, else fp32.  One call of `run_once` is one whole prefill with the
    first-token log-probs; nothing is extrapolated."""

    def __init__(self, args, shape):
        import torch

        from chunkkv_b200.engine.base import BlendConfig, ChunkKV, Placement
        from chunkkv_b200.engine.weights import random_state_dict
        from oracle.blend_oracle import OracleEngine

        torch.set_num_threads(os.cpu_count() or 1)
        self.shape = shape
        self.dtype = self._fastest_dtype()
        # seed-0 random weights, drawn where it is fastest (the GPU when there is one:
        # setup, not timed), held on the host
        gen_dev = "cuda" if torch.cuda.is_available() else "cpu"
        sd = random_state_dict(shape, seed=0, dtype=torch.bfloat16, device=gen_dev)
        sd = {k: v.to("cpu", self.dtype) for k, v in sd.items()}
        self.eng = OracleEngine(shape, sd, dtype=self.dtype)
        del sd
        chunks, order, query = make_request(shape.vocab, args.chunks, args.chunk_len, args.query_len, 0)
        H, D, L = shape.n_kv, shape.head_dim, shape.n_layers
        g = torch.Generator().manual_seed(1)
        tokens, pl = [], []
        for c in order:  # cached K/V of N(0, 1) scale, like post-RoPE keys and values
            ck = ChunkKV([torch.randn((1, H, args.chunk_len, D), generator=g).to(self.dtype) for _ in range(L)],
                         [torch.randn((1, H, args.chunk_len, D), generator=g).to(self.dtype) for _ in range(L)],
                         c * args.chunk_len)
            pl.append(Placement(ck, len(tokens)))
            tokens += chunks[c]
        self.tokens, self.pl = tokens + query, pl
        self.ratio = args.ratio
        self.cfg = BlendConfig(recompute_ratio=args.ratio, n_sink=args.n_sink)
        self.threads = torch.get_num_threads()

    @staticmethod
    def _fastest_dtype():
        import torch

        a = torch.randn(1024, 2048)
        best, best_t = torch.float32, float("inf")
        for dt in (torch.float32, torch.bfloat16):
            x, w = a.to(dt), a.to(dt)
            torch.nn.functional.linear(x, w)
            t0 = time.perf_counter()
            for _ in range(3):
                torch.nn.functional.linear(x, w)
            t = time.perf_counter() - t0
            if t < best_t:
                best, best_t = dt, t
        return best

    def run_once(self) -> float:
        """Seconds of one blend prefill with its first-token log-probs."""
        t0 = time.perf_counter()
        res = self.eng.prefill(self.tokens, self.pl, self.cfg)
        self.eng.last_logprobs(res)
        self.n_selected = int(len(res.keep_abs))
        return time.perf_counter() - t0

    @property
    def dtype_name(self) -> str:
        return "bf16" if str(self.dtype).endswith("bfloat16") else "f32"

    def describe(self, reps: int) -> str:
        return (f"oracle port of TorchEngine.prefill (timed equal to the reference's own on a shared CPU "
                f"request) on the host CPU, {self.dtype_name}, all {self.shape.n_layers} layers of the same "
                f"request (N={len(self.tokens)}, {self.ratio:.0%} recompute, {self.n_selected} rows recomputed "
                f"past layer 1), seed-0 random weights; median of {reps} prefills after one warm-up")


def cpu_sample(args, shape, reps: int = 2) -> dict:
    s = CpuSample(args, shape)
    s.run_once()  # warm-up
    t = statistics.median(s.run_once() for _ in range(reps))
    return {"value": round(len(s.tokens) / t, 2), "unit": "tokens/s", "cores": s.threads, "kind": "port",
            "dtype": s.dtype_name, "ttft_ms": round(t * 1e3, 1), "sample": s.describe(reps)}


# ------------------------------------------------------------------ ours
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from chunkkv_b200 import _lib, ops
    from chunkkv_b200.engine.base import BlendConfig, Placement
    from chunkkv_b200.engine.torch_engine import TorchEngine
    from chunkkv_b200.engine.weights import SHAPES, random_packed
    from chunkkv_b200.store.keys import LookupKey
    from chunkkv_b200.store.kvstore import Entry, KVStore
    from chunkkv_b200.types import TrustLevel

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        nccl_init_logging()
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    shape = SHAPES[args.shape]
    weights = random_packed(shape, seed=0, device=dev)
    eng = TorchEngine.from_packed(weights)
    chunks, order, query = make_request(shape.vocab, args.chunks, args.chunk_len, args.query_len,
                                        request_seed(rank))
    # untimed setup: the chunks' K/V from a prefill in the original order, into the paged store
    first = eng.prefill(sum(chunks, []))
    store = KVStore(budget_bytes=2 * args.chunks * args.chunk_len * shape.kv_bytes_per_token)
    paged = []
    for i in range(args.chunks):
        key = LookupKey.build(chunks[i], shape.name, None)
        store.put(key, Entry(first.chunk(i * args.chunk_len, (i + 1) * args.chunk_len), "bench", f"c{i}",
                             TrustLevel.SYSTEM))
        paged.append(store.get(key)[0].kv)
    del first
    torch.cuda.empty_cache()
    tokens, pl = [], []
    for c in order:
        pl.append(Placement(paged[c], len(tokens)))
        tokens += chunks[c]
    tokens += query
    N = len(tokens)
    cfg = BlendConfig(recompute_ratio=args.ratio, n_sink=args.n_sink)

    def step(c=cfg):
        return eng.prefill(tokens, pl, c)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _lib.check_device()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-timed region: K prefills, inputs resident in HBM
    stream = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    barrier()
    torch.cuda.synchronize()
    phys = physical_index(local)
    with ClockSampler(phys) as clk:
        ev[0].record(stream)
        for i in range(args.steps):
            res = step()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
    barrier()
    step_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    total_ms = max_over_ranks(ev[0].elapsed_time(ev[-1]), dev)
    stats = res.stats

    # ---- the same K steps again with an event pair around every launch: per-kernel
    # times for the roofline and the launch count (not part of the timed value).  A device
    # sleep before each pair keeps the GPU from waiting on the host inside the pair.
    with ops.LaunchTimer(gate_us=KERNEL_GATE_US) as timer:
        for i in range(args.steps):
            step()
        torch.cuda.synchronize()
    kern = timer.summary()
    launches = sum(d["kernels"] for d in kern.values())

    # ---- e2e: the public API with host buffers (token list in, log-probs out),
    # timed by device events that bracket the host work, H2D, kernels and D2H
    barrier()
    torch.cuda.synchronize()
    for _ in range(2):  # untimed: the public path's first calls (host buffers, log-prob readback)
        lp = eng.last_logprobs(eng.prefill(tokens, pl, cfg))
    barrier()
    e2e_ms = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        r = eng.prefill(tokens, pl, cfg)
        lp = eng.last_logprobs(r)  # blocking D2H of the log-probs
        e1.record(stream)
        e1.synchronize()
        e2e_ms.append(e0.elapsed_time(e1))
    e2e_total = max_over_ranks(sum(e2e_ms), dev) * 1e-3
    h2d = eng.last_h2d_bytes
    d2h = eng.last_d2h_bytes + lp.nbytes

    extra = {}
    for rs in [float(x) for x in args.extra_ratios.split(",") if x]:
        c2 = BlendConfig(recompute_ratio=rs, n_sink=args.n_sink)
        step(c2)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(3, args.steps // 4)
        e0.record()
        for _ in range(n):
            step(c2)
        e1.record()
        torch.cuda.synchronize()
        extra[f"{rs:.2f}"] = round(e0.elapsed_time(e1) / n, 3)

    _lib.check_device()
    n_selected = int(len(res.selected))
    tp_out = tp_chk = None
    if world > 1:
        # the collective path: config 5 (32B, 32k tokens) split by KV head over the same
        # ranks, bounded to a few steps, and its parity against one GPU
        del step, eng, weights, store, paged, pl, res, r
        torch.cuda.empty_cache()
        barrier()
        tp_out = tp_leg(world, rank, dev, "qwen2.5-32b", 64, 512, 128, 0.15, 4, steps=max(3, min(args.steps, 5)),
                        warmup=2, fused=True, clocks_index=phys)
        tp_chk = tp_check(world, rank, dev)
        dist.destroy_process_group()
    if rank != 0:
        return

    pk, pk_kind = peaks()
    gemm_names = ("ckv_linear", "ckv_linear_residual", "ckv_linear_swiglu", "ckv_qkv_rope")
    g_ms = sum(kern[n]["ms"] for n in gemm_names if n in kern)
    g_fl = sum(kern[n]["flops"] for n in gemm_names if n in kern)
    busy = sum(d["ms"] for d in kern.values())
    roof = dominant_roofline(timer, pk, pk_kind, shape)
    roof["gemm_family"] = {"kernels": "qkv+rope, o_proj+residual, gate/up+swiglu, down+residual",
                           "achieved": round(g_fl / (g_ms * 1e-3) / 1e12, 1) if g_ms else 0.0,
                           "frac": round(g_fl / (g_ms * 1e-3) / 1e12 / roof["peak"], 4) if g_ms else 0.0,
                           "frac_sustained": round(g_fl / (g_ms * 1e-3) / 1e12 / pk["bf16_tflops_sustained"], 4)
                           if g_ms else 0.0,
                           "frac_burst": round(g_fl / (g_ms * 1e-3) / 1e12 / pk["bf16_tflops"], 4) if g_ms else 0.0,
                           "share_of_busy": round(g_ms / busy, 4) if busy else 0.0}
    kernels = {}
    for name, d in sorted(kern.items(), key=lambda kv: -kv[1]["ms"]):
        e = {"launches": d["launches"], "kernels": d["kernels"], "ms": round(d["ms"], 3),
             "share": round(d["ms"] / busy, 4) if busy else 0}
        if d["flops"] and name != "ckv_gemv":
            tf = d["flops"] / (d["ms"] * 1e-3) / 1e12
            e.update(tflops=round(tf, 1), frac_tensor=round(tf / pk["bf16_tflops_sustained"], 4),
                     frac_tensor_burst=round(tf / pk["bf16_tflops"], 4))
        if d["bytes"]:
            gb = d["bytes"] / (d["ms"] * 1e-3) / 1e9
            e.update(gbs=round(gb, 1), frac_hbm=round(gb / pk["hbm_gbs"], 4),
                     bytes_per_launch=round(d["bytes"] / d["launches"]))
        kernels[name] = e
    ms_step = total_ms / args.steps
    out = {
        "metric": METRIC, "value": round(N * args.steps * world / (total_ms * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init bf16 weights (seed 0), uniform random token ids",
        "config": {"workload": "BASELINE config 3: shuffled multi-chunk blend prefill, 1 request per step per GPU",
                   "model": f"{args.shape} architecture, random init", "tokens": N,
                   "cached_tokens": args.chunks * args.chunk_len, "chunks": f"{args.chunks}x{args.chunk_len}",
                   "query_tokens": args.query_len, "recompute_ratio": args.ratio, "n_sink": args.n_sink,
                   "global_batch": world, "seq_len": N, "parallelism": f"dp{world} (request replicas)",
                   "l2": "inputs larger than L2 every step (15.2 GB weights, 0.6 GB cached K/V pages)"},
        "ttft_ms_p50": round(statistics.median(step_ms), 3), "ttft_ms_p95": round(sorted(step_ms)[
            min(len(step_ms) - 1, int(0.95 * len(step_ms)))], 3),
        "ttft_ms_by_ratio": {f"{args.ratio:.2f}": round(statistics.median(step_ms), 3), **extra},
        "selected_tokens": n_selected, "recomputed_cached_tokens": stats["recomputed_cached_tokens"],
        "prefill_token_equiv": stats["prefill_token_equiv"],
        "e2e": {"value": round(N * args.steps * world / e2e_total, 1), "unit": "tokens/s",
                "ttft_ms_p50": round(statistics.median(e2e_ms), 3),
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "api": "TorchEngine.prefill(list[int], placements from the paged store) + last_logprobs"},
        "roofline": roof, "kernels": kernels, "kernel_timing": KERNEL_TIMING, "gpu_launches": int(launches),
        "gpu_busy_ms_per_step": round(busy / args.steps, 3),
        "clocks": clk.summary(),
    }
    if tp_out is not None:
        top = dict(sorted(tp_out["kernels"].items(), key=lambda kv: -kv[1]["ms"])[:6])
        out["tp"] = {k: tp_out[k] for k in ("metric", "value", "unit", "ttft_ms_p50", "ms_per_step", "steps",
                                            "exchange_us", "selected_tokens", "e2e", "roofline", "clocks")}
        out["tp"]["config"] = tp_out["config"]
        out["tp"]["kernels"] = top
        out["tp_check"] = tp_chk
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_sample(args, shape)
    print(json.dumps(out), flush=True)


# DRAM bytes (read + write) of one ckv_linear_swiglu launch at the selected-row shape
# (M = 938, N = 2 x 18944, K = 3584), measured by ncu (dram__bytes_read.sum +
# dram__bytes_write.sum, one launch of `bench.py --kernel-case swiglu`, clocks not
# locked): 305.3 MB, against 313.8 MB algorithmic (the 271.6 MB weight, the 6.7 MB
# activation read and the 35.5 MB output write; part of the output write was still
# in L2 when the launch ended).
SWIGLU_M938_TRAFFIC = 305.3e6


def dominant_roofline(timer, pk, pk_kind, shape):
    """Roofline of the step's dominant kernel, the gate/up GEMM with the SwiGLU
    epilogue, over its launches at the selected-row shape (every layer after the
    first); achieved = algorithmic FLOPs per launch / mean CUDA-event duration."""
    groups: dict[float, list[float]] = {}
    for name, flops, _nb, e0, e1 in timer.records:
        if name == "ckv_linear_swiglu":
            groups.setdefault(flops, []).append(e0.elapsed_time(e1))
    if not groups:
        return {"bound": "tensor", "achieved": 0.0, "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                "frac": 0.0, "traffic": None}
    flops, times = max(groups.items(), key=lambda kv: len(kv[1]))
    ms = statistics.mean(times)
    achieved = flops / (ms * 1e-3) / 1e12
    m_rows = round(flops / (4.0 * shape.inter * shape.hidden))
    # A launch timed after a device sleep runs alone, like the short cuBLAS run of the burst
    # peak, so that is its denominator; without the sleep the launches run back to back
    # inside the step, like the sustained run.
    key = "bf16_tflops" if getattr(timer, "gate_cycles", 0) else "bf16_tflops_sustained"
    return {"kernel": "ckv_linear_swiglu (tcgen05 gate/up GEMM + SwiGLU epilogue), layers >= 1",
            "bound": "tensor", "achieved": round(achieved, 1), "peak": pk[key],
            "unit": "TFLOP/s", "frac": round(achieved / pk[key], 4), "peak_source": f"{pk_kind} {key}",
            "peak_burst": pk["bf16_tflops"], "frac_burst": round(achieved / pk["bf16_tflops"], 4),
            "peak_sustained": pk["bf16_tflops_sustained"],
            "frac_sustained": round(achieved / pk["bf16_tflops_sustained"], 4),
            "peak_sustained_sm_mhz": pk.get("sustained_sm_mhz"),
            "launches": len(times), "rows": m_rows,
            "flops_per_launch": round(flops), "ms_per_launch": round(ms, 4),
            "traffic": SWIGLU_M938_TRAFFIC if (m_rows == 938 and shape.name == "qwen2.5-7b") else None,
            "traffic_note": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at M = 938"}


def tp_order(n_chunks: int, chunk_len: int, max_shift: int, seed: int) -> list[int]:
    """Seeded order of the chunks for the TP workload: shuffled within blocks of
    max_shift // chunk_len chunks, so every chunk moves by at most max_shift tokens."""
    rng = random.Random(seed)
    blk = max(2, max_shift // chunk_len)
    order = []
    for b in range(0, n_chunks, blk):
        part = list(range(b, min(b + blk, n_chunks)))
        rng.shuffle(part)
        order += part
    return order


def tp_leg(world: int, rank: int, dev, shape_name: str, n_chunks: int, chunk_len: int, query_len: int,
           ratio: float, n_sink: int, steps: int, warmup: int, fused: bool, clocks_index=None) -> dict | None:
    """Config 5 on the initialised process group: one shuffled request split over all
    ranks by KV head (tensor parallel; exchanges after o_proj and down_proj over NVLink
    peer memory when `fused`, else NCCL all-reduce; NCCL all-reduce of the layer-1
    scores).  Returns the measurement on rank 0 (None on the others)."""
    import torch
    import torch.distributed as dist

    from chunkkv_b200 import _lib, ops
    from chunkkv_b200.engine.base import BlendConfig, Placement
    from chunkkv_b200.engine.torch_engine import TorchEngine
    from chunkkv_b200.engine.tp import TensorParallel
    from chunkkv_b200.engine.weights import SHAPES, random_packed
    from chunkkv_b200.store.keys import LookupKey
    from chunkkv_b200.store.kvstore import Entry, KVStore
    from chunkkv_b200.types import TrustLevel

    tp = TensorParallel(fused=fused) if world > 1 else None
    shape = SHAPES[shape_name]
    weights = random_packed(shape, seed=0, device=dev, tp_rank=rank, tp_size=world)
    eng = TorchEngine.from_packed(weights, tp=tp)
    loc = weights.shape
    # every rank serves the same request (its heads of it)
    chunks, _, query = make_request(shape.vocab, n_chunks, chunk_len, query_len, request_seed(0))
    order = tp_order(n_chunks, chunk_len, 16384, request_seed(0))
    first = eng.prefill(sum(chunks, []))
    store = KVStore(budget_bytes=2 * n_chunks * chunk_len * loc.kv_bytes_per_token)
    paged = []
    for i in range(n_chunks):
        key = LookupKey.build(chunks[i], shape.name, None)
        store.put(key, Entry(first.chunk(i * chunk_len, (i + 1) * chunk_len), "bench", f"c{i}",
                             TrustLevel.SYSTEM))
        paged.append(store.get(key)[0].kv)
    del first
    torch.cuda.empty_cache()
    tokens, pl = [], []
    for c in order:
        pl.append(Placement(paged[c], len(tokens)))
        tokens += chunks[c]
    tokens += query
    N = len(tokens)
    max_delta = max(abs(p.start - p.chunk.start) for p in pl)
    cfg = BlendConfig(recompute_ratio=ratio, n_sink=n_sink)

    def step():
        return eng.prefill(tokens, pl, cfg)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    _lib.check_device()
    stream = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(clocks_index if clocks_index is not None else dev.index) as clk:
        ev[0].record(stream)
        for i in range(steps):
            res = step()
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
    barrier()
    step_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    total_ms = max_over_ranks(ev[0].elapsed_time(ev[-1]), dev)
    with ops.LaunchTimer() as timer:
        for i in range(steps):
            step()
        torch.cuda.synchronize()
    kern = timer.summary()
    barrier()
    torch.cuda.synchronize()
    for _ in range(2):  # untimed: the public path's first calls (host buffers, log-prob readback)
        lp = eng.last_logprobs(eng.prefill(tokens, pl, cfg))
    barrier()
    e2e_ms = []
    for _ in range(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        r = eng.prefill(tokens, pl, cfg)
        lp = eng.last_logprobs(r)
        e1.record(stream)
        e1.synchronize()
        e2e_ms.append(e0.elapsed_time(e1))
    e2e_total = max_over_ranks(sum(e2e_ms), dev) * 1e-3
    _lib.check_device()
    barrier()
    if tp is not None and tp._exchange is not None:
        tp._exchange.close()
    n_sel = int(len(res.selected))
    recomputed = res.stats["recomputed_cached_tokens"]
    h2d, d2h = int(eng.last_h2d_bytes), int(eng.last_d2h_bytes + lp.nbytes)
    del eng, res, r, store, paged, pl, weights
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    pk, pk_kind = peaks()
    busy = sum(d["ms"] for d in kern.values())
    kernels = {}
    for name, d in sorted(kern.items(), key=lambda kv: -kv[1]["ms"]):
        e = {"launches": d["launches"], "kernels": d["kernels"], "ms": round(d["ms"], 3),
             "share": round(d["ms"] / busy, 4) if busy else 0}
        if d["flops"] and name != "ckv_gemv":
            tf = d["flops"] / (d["ms"] * 1e-3) / 1e12
            e.update(tflops=round(tf, 1), frac_tensor=round(tf / pk["bf16_tflops_sustained"], 4),
                     frac_tensor_burst=round(tf / pk["bf16_tflops"], 4))
        if d["bytes"]:
            gb = d["bytes"] / (d["ms"] * 1e-3) / 1e9
            if name in ("nccl_all_reduce", "ckv_reduce_add_gather"):
                e.update(bus_gbs=round(gb, 1), frac_nvlink=round(gb / 770.0, 4),
                         bus_bytes_per_launch=round(d["bytes"] / d["launches"]),
                         us_per_launch=round(1e3 * d["ms"] / d["launches"], 2))
            else:
                e.update(gbs=round(gb, 1), frac_hbm=round(gb / pk["hbm_gbs"], 4),
                         bytes_per_launch=round(d["bytes"] / d["launches"]))
        kernels[name] = e
    gemm_names = ("ckv_linear", "ckv_linear_residual", "ckv_linear_swiglu", "ckv_qkv_rope", "ckv_linear_partial")
    g_ms = sum(kern[n]["ms"] for n in gemm_names if n in kern)
    g_fl = sum(kern[n]["flops"] for n in gemm_names if n in kern)
    g_tf = g_fl / (g_ms * 1e-3) / 1e12 if g_ms else 0.0
    exch = kernels.get("ckv_reduce_add_gather") or kernels.get("nccl_all_reduce")
    return {
        "metric": f"blend-prefill tokens/s ({shape_name} shape, tensor parallel over {world} GPU(s), "
                  f"{n_chunks}x{chunk_len} shuffled cached chunks + {query_len}-token query)",
        "value": round(N * steps / (total_ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(total_ms / steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init bf16 weights (seed 0, sharded per rank), uniform random token ids",
        "config": {"workload": "BASELINE config 5: one shuffled 32k-token blend prefill split by KV head",
                   "model": f"{shape_name} architecture, random init", "tokens": N,
                   "cached_tokens": n_chunks * chunk_len, "chunks": f"{n_chunks}x{chunk_len}",
                   "max_abs_delta": max_delta, "query_tokens": query_len, "recompute_ratio": ratio,
                   "n_sink": n_sink, "parallelism": f"tp{world} (KV heads {loc.n_kv} per rank)",
                   "tp_exchange": ("none (one GPU)" if tp is None else
                                   "partial rows over NVLink peer memory (ckv_linear_partial + "
                                   "ckv_reduce_add_gather)" if fused else "NCCL all-reduce"),
                   "l2": "inputs larger than L2 every step (weights and cached K/V pages)"},
        "ttft_ms_p50": round(statistics.median(step_ms), 3),
        "selected_tokens": n_sel, "recomputed_cached_tokens": recomputed,
        "exchange_us": exch.get("us_per_launch") if exch else None,
        "e2e": {"value": round(N * steps / e2e_total, 1), "unit": "tokens/s",
                "ttft_ms_p50": round(statistics.median(e2e_ms), 3),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"kernel": "tcgen05 GEMMs (all entry points)", "bound": "tensor",
                     "achieved": round(g_tf, 1), "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": round(g_tf / pk["bf16_tflops_sustained"], 4),
                     "peak_source": f"{pk_kind} bf16_tflops_sustained", "traffic": None},
        "kernels": kernels, "gpu_launches": int(sum(d["kernels"] for d in kern.values())),
        "gpu_busy_ms_per_step": round(busy / steps, 3), "clocks": clk.summary(),
    }


def tp_check(world: int, rank: int, dev, n_layers: int = 3) -> dict:
    """Tensor-parallel parity on the hardware the bench runs on (product code only): a
    truncated 32B model (n_layers layers; hidden, heads and MLP at full size) split by
    KV head over all ranks, against a one-GPU engine with the same weights on every
    rank, both exchanges, both blending the one-GPU engine's cached chunks.  Per rank: first-token logit KL(one GPU || split), the
    selection from the split run's all-reduced layer-1 scores equal to the split run's
    kept positions (the one-GPU selection kernel), this rank's blended K/V heads (moved
    positions neither run recomputed) against the same heads of the one-GPU cache.
    Rank 0 returns the worst case over ranks."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from chunkkv_b200 import _lib, ops
    from chunkkv_b200.engine.base import BlendConfig, ChunkKV, Placement, plan_arrays
    from chunkkv_b200.engine.torch_engine import TorchEngine
    from chunkkv_b200.engine.tp import TensorParallel
    from chunkkv_b200.engine.weights import SHAPES, pack, random_state_dict

    shape = SHAPES["qwen2.5-32b"].truncated(n_layers)
    sd = random_state_dict(shape, seed=0, dtype=torch.bfloat16, device=dev)  # same values on every rank
    single = TorchEngine.from_packed(pack(shape, sd, device=dev))
    chunks, order, query = make_request(shape.vocab, 8, 256, 64, request_seed(0))
    cfg = BlendConfig(recompute_ratio=0.15, n_sink=4)

    def blend(eng, cached):
        toks, pl = [], []
        for c in order:
            pl.append(Placement(cached[c], len(toks)))
            toks += chunks[c]
        toks += query
        return toks, pl, eng.prefill(toks, pl, cfg)

    # both runs blend the same cached chunks (the one-GPU engine's first prefill; each
    # rank receives its own KV heads of them), so K/V at moved positions is a pure gather
    # and re-RoPE on both sides
    first = single.prefill(sum(chunks, []))
    cached1 = [first.chunk(i * 256, (i + 1) * 256) for i in range(8)]
    tokens, pl1, ref = blend(single, cached1)
    K1, V1 = ref.cache
    ref_sel = ref.selected.cpu().numpy()
    out = {"layers": n_layers, "tokens": len(tokens), "ranks": world}
    worst = {"kl": 0.0, "kv_rel": 0.0, "selection_exact": True, "ranks_agree": True}
    for fused in (True, False):
        tp = TensorParallel(fused=fused)
        eng = TorchEngine.from_packed(pack(shape, sd, device=dev, tp_rank=rank, tp_size=world), tp=tp)
        hl = shape.n_kv // world
        hs = slice(rank * hl, (rank + 1) * hl)
        mine = [ChunkKV([k[:, hs].contiguous() for k in ck.keys], [v[:, hs].contiguous() for v in ck.values],
                        ck.start) for ck in cached1]
        _, pl, res = blend(eng, mine)
        torch.cuda.synchronize()
        N = len(tokens)
        sel = res.selected.cpu().numpy()
        # the one-GPU selection kernel on the split run's all-reduced scores
        ws = ops.SelectWorkspace(N, len(pl), dev)
        summed = eng._ws  # the split run's workspace holds the all-reduced scores
        plan = plan_arrays(N, pl, cfg.n_sink)
        meta = torch.tensor([[p.start, p.chunk.length, int(round(cfg.recompute_ratio * p.chunk.length)), 0]
                             for p in pl], dtype=torch.int32, device=dev)
        ops.select_from_scores(summed.diff[:N], summed.norm[:N], torch.from_numpy(plan.pos_flags()).to(dev),
                               meta, None, ws)
        n = int(ws.counts[0])
        exact = bool(np.array_equal(ws.keep_abs[:n].cpu().numpy(), sel))
        p_ref = torch.log_softmax(ref.logits[-1].float(), -1)
        p_tp = torch.log_softmax(res.logits[-1].float(), -1)
        kl = float((p_ref.exp() * (p_ref - p_tp)).sum())
        # blended K/V (moved by re-RoPE, recomputed by neither run) under the bf16 bar;
        # the recomputed positions follow the residual stream, whose split sums round
        # differently, and are reported beside it
        moved = plan.cached.copy()
        moved[sel] = False
        moved[ref_sel] = False
        both = np.zeros(N, bool)
        both[np.intersect1d(sel, ref_sel)] = True
        K2, V2 = res.cache

        def rel(a, b):
            a, b = a.float(), b.float()
            return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))

        def kv_err(mask):
            m = torch.from_numpy(mask).to(dev)
            return max(rel(K2[:, :, m], K1[:, hs][:, :, m]), rel(V2[:, :, m], V1[:, hs][:, :, m]))

        kv = kv_err(moved)
        kv_recomputed = kv_err(both)
        # the replicated selection is identical on every rank
        selt = torch.tensor(sel.astype(np.int64), device=dev)
        lens = torch.tensor([selt.numel()], device=dev)
        lmax = lens.clone()
        dist.all_reduce(lmax, op=dist.ReduceOp.MAX)
        lmin = lens.clone()
        dist.all_reduce(lmin, op=dist.ReduceOp.MIN)
        agree = bool(lmax.item() == lmin.item())
        if agree:
            hi, lo = selt.clone(), selt.clone()
            dist.all_reduce(hi, op=dist.ReduceOp.MAX)
            dist.all_reduce(lo, op=dist.ReduceOp.MIN)
            agree = bool(torch.equal(hi, lo))
        vals = torch.tensor([kl, kv, 0.0 if exact else 1.0, 0.0 if agree else 1.0, kv_recomputed],
                            dtype=torch.float64, device=dev)
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        out[f"{'peer' if fused else 'nccl'}_exchange"] = {"kl_max": float(vals[0]), "kv_rel_max": float(vals[1]),
                                                          "selection_exact": bool(vals[2] == 0),
                                                          "ranks_agree": bool(vals[3] == 0),
                                                          "kv_rel_max_recomputed": float(vals[4])}
        worst["kl"] = max(worst["kl"], float(vals[0]))
        worst["kv_rel"] = max(worst["kv_rel"], float(vals[1]))
        worst["selection_exact"] &= bool(vals[2] == 0)
        worst["ranks_agree"] &= bool(vals[3] == 0)
        if tp._exchange is not None:
            tp._exchange.close()
        del eng, res
    _lib.check_device()
    del single, ref, sd, first, cached1
    torch.cuda.empty_cache()
    out["pass"] = bool(worst["kl"] <= 1e-3 and worst["kv_rel"] <= 1e-2 and worst["selection_exact"]
                       and worst["ranks_agree"])
    out["criteria"] = ("first-token KL <= 1e-3, blended (moved) K/V max rel err <= 1e-2, selection exact given "
                       "the summed scores, ranks agree")
    return out


def run_tp(args):
    """Config 5 alone (`--workload tp`): prints the tensor-parallel line."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        nccl_init_logging()
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    out = tp_leg(world, rank, dev, args.shape, args.chunks, args.chunk_len, args.query_len, args.ratio,
                 args.n_sink, args.steps, args.warmup, args.tp_exchange == "peer", physical_index(local))
    if world > 1:
        dist.destroy_process_group()
    if out is not None:
        out["cpu_baseline"] = None
        out["cpu_baseline_note"] = "infeasible on the host at 32B x 32k tokens"
        print(json.dumps(out), flush=True)


def replay_requests(n_req: int, vocab: int, seed: int = 7):
    """Config 4 request stream: a pool of 16 chunks x 256 tokens; each request is a
    distinct 200-token prefix, 6-12 pool chunks sampled without replacement in random
    order, and a 16-token query (the last position must be computed for its logits)."""
    rng = random.Random(seed)
    pool = [[rng.randrange(vocab) for _ in range(256)] for _ in range(16)]
    reqs = []
    for _ in range(n_req):
        prefix = [rng.randrange(vocab) for _ in range(200)]
        picks = rng.sample(range(16), rng.randint(6, 12))
        query = [rng.randrange(vocab) for _ in range(16)]
        reqs.append((prefix, picks, query))
    return pool, reqs


def lpt_assign(sizes: list[int], world: int) -> list[list[int]]:
    """Longest-processing-time assignment of requests (by token count) to ranks."""
    loads = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(sizes)), key=lambda i: -sizes[i]):
        r = min(range(world), key=lambda r: loads[r])
        out[r].append(i)
        loads[r] += sizes[i]
    return [sorted(o) for o in out]


def run_replay(args):
    """Config 4: requests over a shared chunk pool, data parallel over the GPUs (each
    rank warms its own pool copy in its own paged store and serves its LPT share).
    Per request, like ChunkReuseRuntime.prefill (runtime.py:50-93) with every reusable
    segment blended: store lookups -> blend prefill -> first-token log-probs -> the
    request's chunk segments written back to the store as new variants."""
    import torch
    import torch.distributed as dist

    from chunkkv_b200 import _lib
    from chunkkv_b200.engine.torch_engine import TorchEngine
    from chunkkv_b200.engine.weights import SHAPES, random_packed
    from chunkkv_b200.gate import GateConfig, ReuseGate
    from chunkkv_b200.runtime import ChunkReuseRuntime
    from chunkkv_b200.store.keys import LookupKey, token_hash
    from chunkkv_b200.store.kvstore import Entry, KVStore
    from chunkkv_b200.types import ChunkedRequest, Segment, TrustLevel

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    shape = SHAPES[args.shape]
    eng = TorchEngine.from_packed(random_packed(shape, seed=0, device=dev))
    pool, reqs = replay_requests(args.requests, shape.vocab)
    store = KVStore(budget_bytes=40 << 30, pool_bytes=40 << 30, device=dev)
    warm = eng.prefill(sum(pool, []))
    for i, c in enumerate(pool):
        store.put(LookupKey.build(c, shape.name, None),
                  Entry(warm.chunk(i * 256, (i + 1) * 256), "pool", token_hash([]), TrustLevel.SYSTEM))
    del warm
    sizes = [200 + 256 * len(p) + 16 for _, p, _ in reqs]
    mine = lpt_assign(sizes, world)[rank]
    # policy P3 of the reference's bench/policies.py: every stored chunk is blended at
    # the fixed ratio, lookup keys without the tenant
    gate = ReuseGate(GateConfig(mode="always_blend", ratio_same_context=args.ratio))
    runtime = ChunkReuseRuntime(eng, shape.name, store, gate, provenance=False)

    def request(i) -> ChunkedRequest:
        prefix, picks, query = reqs[i]
        segs = [Segment(0, "system", TrustLevel.SYSTEM, 0, list(prefix), reusable=False)]
        tokens = list(prefix)
        for c in picks:
            segs.append(Segment(len(segs), "tool", TrustLevel.TOOL, len(tokens), pool[c]))
            tokens += pool[c]
        segs.append(Segment(len(segs), "user", TrustLevel.USER, len(tokens), list(query), reusable=False))
        return ChunkedRequest(tokens + list(query), segs, f"tenant{i % 4}", "replay")

    def serve(i):
        out = runtime.prefill(request(i))
        return out.stats["tokens"], eng.last_logprobs(out.result)

    for i in mine[:max(1, args.warmup)]:
        serve(i)
    torch.cuda.synchronize()
    _lib.check_device()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys = int(vis.split(",")[local]) if vis and vis.split(",")[local].strip().isdigit() else local
    ttft, toks = [], 0
    with ClockSampler(phys) as clk:
        t_all0 = torch.cuda.Event(enable_timing=True)
        t_all0.record(stream)
        for i in mine:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            n, _ = serve(i)
            e1.record(stream)
            e1.synchronize()
            ttft.append(e0.elapsed_time(e1))
            toks += n
        t_all1 = torch.cuda.Event(enable_timing=True)
        t_all1.record(stream)
        torch.cuda.synchronize()
    my_ms = t_all0.elapsed_time(t_all1)
    _lib.check_device()
    total_ms = max_over_ranks(my_ms, dev)
    all_ttft, all_toks = [ttft], [toks]
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, (ttft, toks))
        all_ttft = [g[0] for g in gathered]
        all_toks = [g[1] for g in gathered]
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    flat = sorted(x for t in all_ttft for x in t)
    out = {
        "metric": "config-4 replay requests/s (Qwen2.5-7B shape, 16x256 chunk pool, 6-12 chunks per request)",
        "value": round(args.requests / (total_ms * 1e-3), 2), "unit": "requests/s", "n_gpus": world,
        "steps": args.requests, "warmup": max(1, args.warmup), "ms_per_step": round(total_ms / max(1, len(mine)), 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init bf16 weights (seed 0), seeded random prefixes, pool chunks and queries",
        "config": {"workload": "BASELINE config 4: DP replay through ChunkReuseRuntime with policy P3 "
                               "(always_blend gate, provenance off): per request store lookups, gate, blend "
                               "prefill, log-probs and write-back of the chunk segments",
                   "model": f"{args.shape} architecture, random init", "requests": args.requests,
                   "pool": "16x256", "prefix_tokens": 200, "query_tokens": 16, "recompute_ratio": args.ratio,
                   "n_sink": args.n_sink, "store_bytes_per_gpu": 40 << 30,
                   "parallelism": f"dp{world} (requests assigned LPT by token count)"},
        "tokens_per_s": round(sum(all_toks) / (total_ms * 1e-3), 1),
        "ttft_ms_p50": round(statistics.median(flat), 3),
        "ttft_ms_p95": round(flat[min(len(flat) - 1, int(0.95 * len(flat)))], 3),
        "requests_per_gpu": [len(t) for t in all_ttft],
        "e2e": {"value": round(args.requests / (total_ms * 1e-3), 2), "unit": "requests/s",
                "h2d_bytes_per_step": int(eng.last_h2d_bytes), "d2h_bytes_per_step": int(eng.last_d2h_bytes),
                "note": "the timed loop is the public API end to end (host token lists in, log-probs out)"},
        "clocks": clk.summary(),
    }
    print(json.dumps(out), flush=True)


def policy_requests(n_req: int, vocab: int, seed: int = 11):
    """A multi-tenant agent stream at model scale: two agents' system prompts (300
    tokens, SYSTEM), a pool of 12 tool documents (256-512 tokens, TOOL, reusable),
    3-6 documents per request in random order, sometimes after a user turn (which
    lowers the trust floor of what follows), and a 32-64 token user query; four
    tenants.  The shape of the reference's multi-agent traces, with seeded ids."""
    from chunkkv_b200.types import ChunkedRequest, Segment, TrustLevel

    rng = random.Random(seed)

    def toks(k):
        return [rng.randrange(vocab) for _ in range(k)]

    systems = {"agentA": toks(300), "agentB": toks(300)}
    docs = [toks(rng.randrange(256, 513)) for _ in range(12)]
    out = []
    for i in range(n_req):
        ctx = "agentA" if rng.random() < 0.6 else "agentB"
        segs, tokens = [], []

        def add(role, trust, t, reusable=True):
            segs.append(Segment(len(segs), role, trust, len(tokens), list(t), reusable))
            tokens.extend(t)

        add("system", TrustLevel.SYSTEM, systems[ctx])
        if rng.random() < 0.2:
            add("user", TrustLevel.USER, toks(24), reusable=False)
        for d in rng.sample(range(len(docs)), rng.randint(3, 6)):
            add("tool", TrustLevel.TOOL, docs[d])
        add("user", TrustLevel.USER, toks(rng.randint(32, 64)), reusable=False)
        out.append((f"r{i}", ChunkedRequest(tokens, segs, f"tenant{i % 4}", ctx)))
    return out


def run_policies(args):
    """Policies P0-P4 over one engine (the reference's bench/replay.py + report.py,
    policies of bench/policies.py): every request of the stream under each policy,
    P0 first as the reference for KL and greedy agreement; TTFT is wall clock around
    prefill + first-token log-probs, as the reference measures it."""
    import torch

    from chunkkv_b200.engine.torch_engine import TorchEngine
    from chunkkv_b200.engine.weights import SHAPES, random_packed
    from chunkkv_b200.harness import replay_policy, summarize
    from chunkkv_b200.policies import DESCRIPTIONS, POLICIES, build

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = SHAPES[args.shape]
    eng = TorchEngine.from_packed(random_packed(shape, seed=0, device=dev))
    eng.eos = set()  # random weights: always generate max_new tokens
    reqs = policy_requests(args.requests, shape.vocab)
    eng.last_logprobs(eng.prefill(reqs[0][1].tokens))  # warm-up (plans, workspaces)
    ref: dict = {}
    summary = {}
    for pol in POLICIES:
        rt = build(pol, eng, shape.name, budget_bytes=3 << 30, ratio=args.ratio)
        rows = replay_policy(pol, rt, eng, reqs, ref, max_new=args.max_new, sync=torch.cuda.synchronize)
        s = summarize(rows)
        s["tokens"] = int(sum(r["tokens"] for r in rows))
        s["description"] = DESCRIPTIONS[pol]
        summary[pol] = s
        del rt
        torch.cuda.empty_cache()
    p1 = summary["P1"]["ttft_p50"]
    for s in summary.values():
        s["speedup_vs_p1"] = round(p1 / s["ttft_p50"], 3)
        s["ttft_p50_ms"], s["ttft_p95_ms"] = round(s.pop("ttft_p50") * 1e3, 3), round(s.pop("ttft_p95") * 1e3, 3)
    print(json.dumps({
        "metric": "policy replay TTFT p50 under P4 (gate + provenance keys)",
        "value": summary["P4"]["ttft_p50_ms"], "unit": "ms", "n_gpus": 1, "steps": len(reqs),
        "higher_is_better": False, "dtype": "bf16",
        "data": "synthetic: random-init bf16 weights (seed 0), seeded multi-tenant agent stream",
        "config": {"workload": "P0-P4 policy replay (bench/replay.py + report.py of the reference)",
                   "model": f"{args.shape} architecture, random init", "requests": len(reqs),
                   "ratio": args.ratio, "max_new": args.max_new, "store_budget_bytes": 3 << 30},
        "policies": summary,
    }), flush=True)


def run_micro(args):
    """Config 2: the bandwidth-bound kernels at the 7B KV shape (H = 4, D = 128), 28 layers,
    8 chunks x 256 tokens, Delta uniform in [-4096, 4096].  Each kernel runs on enough sets
    of inputs AND outputs, used in turn, that neither are still in L2 when their turn
    comes again; GB/s are the algorithmic bytes (read + write) over the device time per
    launch (CUDA events around a CUDA graph of the launches)."""
    import torch

    from chunkkv_b200 import ops
    from chunkkv_b200.engine.weights import SHAPES
    from chunkkv_b200.store.pages import PAGE_TOKENS, PagePool

    dev = torch.device("cuda", 0)
    shape = SHAPES["qwen2.5-7b"]
    L, H, D = shape.n_layers, shape.n_kv, shape.head_dim
    n_ch, cl = 8, 256
    T = n_ch * cl
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(0)
    inv = shape.rope_theta ** (-torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D)
    rng = random.Random(1)
    deltas = [rng.randint(-4096, 4096) for _ in range(n_ch)]
    pk, pk_kind = peaks()

    def timed(fn, nbytes, reps=None):
        """Device time per launch: `reps` launches captured in one CUDA graph, replayed
        between two events (eager launches of a ~10 µs kernel would time the host's
        launch rate instead of the kernel)."""
        reps = reps or max(3, args.steps)
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(reps):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        ms = e0.elapsed_time(e1) / reps
        gbs = nbytes / (ms * 1e-3) / 1e9
        return {"ms": round(ms, 4), "bytes": int(nbytes), "gbs": round(gbs, 1), "frac_hbm": round(gbs / pk["hbm_gbs"], 4)}

    def sets_for(nbytes):
        """Input/output sets used in turn so that, between two uses of one set, the
        other sets move at least three times the L2 (126 MB): neither the inputs nor
        the outputs of a launch are still in L2 when their turn comes again."""
        return max(2, -(-3 * 126_000_000 // int(nbytes)) + 1)

    out = {}
    # re-RoPE by Delta (TorchEngine.shift_keys), all chunks of all layers in one launch
    rr_bytes = 2.0 * L * n_ch * H * cl * D * 2
    ns = sets_for(rr_bytes)
    keys = [torch.randn((L * n_ch, H, cl, D), generator=g, device=dev).to(bf) for _ in range(ns)]
    shifted = [torch.empty_like(k) for k in keys]
    # context, not this library's kernel: a plain device-to-device copy of the same bytes
    out["reference_copy_same_bytes"] = timed(lambda i: shifted[i % ns].copy_(keys[i % ns]), rr_bytes)
    out["rerope_shift_keys"] = timed(lambda i: ops.shift_keys(keys[i % ns], deltas[0], inv, out=shifted[i % ns]),
                                     rr_bytes)
    out["rerope_shift_keys"]["sets"] = ns
    del keys, shifted
    torch.cuda.empty_cache()
    # paged gather of K (re-roped) and V for all layers, chunks placed at shifted positions
    n_pages = T // PAGE_TOKENS
    g_bytes = 2.0 * 2 * L * H * T * D * 2
    ng = sets_for(g_bytes)
    pools = [PagePool(L, H, D, n_pages, dev) for _ in range(ng)]
    for pool in pools:
        pool.pages.normal_(generator=g)
    table = torch.arange(n_pages, dtype=torch.int32, device=dev)
    order = list(range(n_ch))
    rng.shuffle(order)
    meta = torch.tensor([[c * cl // PAGE_TOKENS, cl, order[c] * cl, deltas[c], 0, L, 0, 0] for c in range(n_ch)],
                        dtype=torch.int32, device=dev)
    kall = [torch.empty((L, H, T, D), dtype=bf, device=dev) for _ in range(ng)]
    vall = [torch.empty_like(k) for k in kall]
    out["gather_paged"] = timed(lambda i: ops.blend_gather_paged(pools[i % ng].pages, table, meta, inv, kall[i % ng],
                                                                 vall[i % ng], 0, L), g_bytes)
    out["gather_paged"]["sets"] = ng
    # store insert (write-back): one chunk of 256 tokens, all layers, from a result cache;
    # every set reads another chunk of a gathered cache and writes other pages
    w_bytes = 2.0 * 2 * L * H * cl * D * 2
    nw = min(ng * n_ch, sets_for(w_bytes))
    big = PagePool(L, H, D, nw * (cl // PAGE_TOKENS), dev)
    ids = [torch.arange(w * (cl // PAGE_TOKENS), (w + 1) * (cl // PAGE_TOKENS), dtype=torch.int32, device=dev)
           for w in range(nw)]

    def src_ptrs(w, kv):
        b, c = divmod(w, n_ch)
        t = (kall if kv == 0 else vall)[b]
        return torch.tensor([t[li, :, c * cl:].data_ptr() for li in range(L)],
                            dtype=torch.int64).view(torch.uint64).to(dev)

    kp = [src_ptrs(w, 0) for w in range(nw)]
    vp = [src_ptrs(w, 1) for w in range(nw)]
    out["scatter_pages_write"] = timed(lambda i: ops.pages_write(big.pages, ids[i % nw], cl, kp[i % nw], vp[i % nw],
                                                                 T * D), w_bytes)
    out["scatter_pages_write"]["sets"] = nw
    del pools, kall, vall, big
    torch.cuda.empty_cache()
    # layer-1 deviation + pooled top-k: fresh = cached + noise on 20 % of tokens
    # (16 input sets used in turn: 8 MiB per launch would otherwise stay in L2)
    n_sets = 16
    Kbs, Vbs, kfs, vfs = [], [], [], []
    for si in range(n_sets):
        Kb = torch.randn((H, T, D), generator=g, device=dev).to(bf)
        Vb = torch.randn((H, T, D), generator=g, device=dev).to(bf)
        kf = Kb.permute(1, 0, 2).reshape(T, H * D).clone()
        vf = Vb.permute(1, 0, 2).reshape(T, H * D).clone()
        noisy = torch.rand(T, generator=g, device=dev) < 0.2
        kf[noisy] = (kf[noisy].float() + 0.05 * torch.randn(kf[noisy].shape, generator=g, device=dev)).to(bf)
        Kbs.append(Kb), Vbs.append(Vb), kfs.append(kf), vfs.append(vf)
    active = torch.arange(T, dtype=torch.int32, device=dev)
    flags = torch.ones(T, dtype=torch.uint8, device=dev)
    for c in range(n_ch):
        flags[c * cl:c * cl + 4] |= 2
    smeta = torch.tensor([[c * cl, cl, 38, 0] for c in range(n_ch)], dtype=torch.int32, device=dev)
    ws = ops.SelectWorkspace(T, n_ch, dev)
    out["deviation_select_fused"] = timed(
        lambda i: ops.deviation_select(kfs[i % n_sets], vfs[i % n_sets], Kbs[i % n_sets], Vbs[i % n_sets], active,
                                       flags, smeta, None, ws),
        4.0 * T * H * D * 2 + 8.0 * T)
    out["select_from_scores"] = timed(lambda i: ops.select_from_scores(ws.diff[:T], ws.norm[:T], flags, smeta, None, ws),
                                      8.0 * T)
    n_sel = int(ws.counts[0])
    res = {"metric": "config-2 K/V bandwidth kernels (7B KV shape, 28 layers, 8 chunks x 256 tokens)",
           "unit": "GB/s", "n_gpus": 1, "higher_is_better": True, "peak": pk["hbm_gbs"],
           "peak_source": f"{pk_kind} hbm_gbs", "selected_tokens": n_sel,
           "data": "synthetic: N(0,1) bf16 K/V, seeded deltas and noise",
           "timing": "CUDA events around one CUDA graph of `steps` launches per kernel", "kernels": out}
    print(json.dumps(res), flush=True)


def run_decode(args):
    """Greedy decode after the config-3 blend prefill (TorchEngine.generate,
    torch_engine.py:180-198): per token, 28 layers of m = 1 projections (fused GEMV
    kernels) and attention over the blended cache, then the lm_head GEMV.  Reports ms per
    token and the weight bytes streamed per token against the HBM peak."""
    import torch

    from chunkkv_b200.engine.base import BlendConfig, Placement
    from chunkkv_b200.engine.torch_engine import TorchEngine
    from chunkkv_b200.engine.weights import SHAPES, random_packed

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = SHAPES[args.shape]
    weights = random_packed(shape, seed=0, device=dev)
    eng = TorchEngine.from_packed(weights)
    eng.eos = set()  # random weights: decode the full count
    chunks, order, query = make_request(shape.vocab, args.chunks, args.chunk_len, args.query_len, request_seed(0))
    first = eng.prefill(sum(chunks, []))
    tokens, pl = [], []
    for c in order:
        pl.append(Placement(first.chunk(c * args.chunk_len, (c + 1) * args.chunk_len), len(tokens)))
        tokens += chunks[c]
    tokens += query
    res = eng.prefill(tokens, pl, BlendConfig(recompute_ratio=args.ratio, n_sink=args.n_sink))
    n_new = max(8, args.steps)
    eng.generate(res, max(4, args.warmup))
    torch.cuda.synchronize()

    def timed(n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        toks = eng.generate(res, n)
        e1.record()
        torch.cuda.synchronize()
        return toks, e0.elapsed_time(e1)

    # Each generate call runs its first step eagerly and captures one CUDA graph for the
    # rest; the steady-state time per token is the difference of two call lengths (the
    # median of three calls each, since the capture time varies from call to call).
    shorts = [timed(8) for _ in range(3)]
    longs = [timed(n_new + 8) for _ in range(3)]
    short, ms_short = shorts[0][0], statistics.median(t for _, t in shorts)
    out, ms_long = longs[0][0], statistics.median(t for _, t in longs)
    ms_tok = (ms_long - ms_short) / (len(out) - len(short))
    pk, pk_kind = peaks()
    wbytes = weights.nbytes() - weights.embed.numel() * 2 + (weights.lm_head.numel() * 2 if shape.tied else 0)
    gbs = wbytes / (ms_tok * 1e-3) / 1e9
    print(json.dumps({
        "metric": "greedy decode tokens/s after the config-3 blend prefill (one request)",
        "value": round(1e3 / ms_tok, 2), "unit": "tokens/s", "n_gpus": 1, "steps": len(out) - len(short),
        "ms_per_step": round(ms_tok, 4), "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic: random-init bf16 weights (seed 0)",
        "config": {"workload": "decode after config 3", "model": f"{args.shape} architecture, random init",
                   "context_tokens": len(tokens), "new_tokens": len(out)},
        "ms_per_token_with_capture": round(ms_long / len(out), 4),
        "note": "ms_per_step = (time of a generate call of n + 8 tokens - one of 8) / n: the per-call "
                "eager first step and graph capture cancel",
        "weight_bytes_per_token": int(wbytes), "weight_gbs": round(gbs, 1),
        "frac_hbm": round(gbs / pk["hbm_gbs"], 4), "peak_source": f"{pk_kind} hbm_gbs"}), flush=True)


def run_reference(args):
    """CPU reference arm: the oracle port of the reference path on the host cores, one
    whole prefill of the bench's request per step (all layers, nothing extrapolated).
    At most `--warmup` (capped at 2) warm-up prefills, then `--steps` timed ones, cut
    short once about two minutes of timed prefills have run; the line says how many."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    from chunkkv_b200.engine.weights import SHAPES

    shape = SHAPES[args.shape]
    s = CpuSample(args, shape)
    for _ in range(max(1, min(args.warmup, 2))):
        s.run_once()
    times = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        times.append(s.run_once())
        if time.perf_counter() - t0 > 120.0:
            break
    ttft = statistics.median(times)
    v = len(s.tokens) / ttft
    cb = {"value": round(v, 2), "unit": "tokens/s", "cores": s.threads, "kind": "port", "dtype": s.dtype_name,
          "ttft_ms": round(ttft * 1e3, 1), "sample": s.describe(len(times))}
    out = {"impl": "reference", "metric": METRIC, "value": round(v, 2), "unit": "tokens/s",
           "n_gpus": args.gpus, "steps": len(times), "steps_requested": args.steps, "warmup": args.warmup,
           "ms_per_step": round(1e3 * statistics.mean(times), 1), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": s.dtype_name, "data": "synthetic",
           "config": {"workload": "BASELINE config 3 request on the host CPU (every layer, see cpu_baseline)",
                      "model": f"{args.shape} architecture", "tokens": len(s.tokens)},
           "cpu_baseline": cb,
           "e2e": {"value": round(v, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def run_kernel_case(args):
    """One kernel at the shape it has in the 7B bench (layers >= 2: 938 active tokens),
    launched `steps` times after `warmup` launches; prints ms per launch.  Operands
    are larger than L2 where the real launch's are (weights, cache pages)."""
    import torch

    from chunkkv_b200 import ops
    from chunkkv_b200.engine.weights import SHAPES, interleave_gate_up

    shape = SHAPES[args.shape]
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    bf = torch.bfloat16
    M, N = 938, args.chunks * args.chunk_len + args.query_len
    hid, H, Hq, D = shape.hidden, shape.n_kv, shape.n_heads, shape.head_dim

    def rnd(*s, scale=0.02):
        return (torch.randn(s, generator=g, device=dev) * scale).to(bf)

    x = rnd(M, hid, scale=1.0)
    pos = torch.randperm(N, generator=g, device=dev)[:M].sort().values.to(torch.int32)
    kernel_bytes = None  # set by the bandwidth-bound cases: algorithmic bytes per launch
    if args.kernel_case == "swiglu":
        w, out = rnd(2 * shape.inter, hid), torch.empty((M, shape.inter), dtype=bf, device=dev)
        fn = lambda: ops.linear_swiglu(x, w, out)  # noqa: E731
    elif args.kernel_case == "oproj":
        a, w, h = rnd(M, Hq * D, scale=1.0), rnd(hid, Hq * D), rnd(M, hid, scale=1.0)
        fn = lambda: ops.linear_residual(a, w, h)  # noqa: E731
    elif args.kernel_case == "decode_swiglu":  # one decode row through the fused GEMV
        w, out = rnd(2 * shape.inter, hid), torch.empty((1, shape.inter), dtype=bf, device=dev)
        x1 = x[:1].contiguous()
        fn = lambda: ops.gemv_swiglu(x1, w, out)  # noqa: E731
    elif args.kernel_case == "decode_down":  # one decode row through the residual GEMV (k = inter)
        a1, w, h1 = rnd(1, shape.inter, scale=1.0), rnd(hid, shape.inter), rnd(1, hid, scale=1.0)
        fn = lambda: ops.gemv_residual(a1, w, h1)  # noqa: E731
    elif args.kernel_case == "down":
        a, w, h = rnd(M, shape.inter, scale=1.0), rnd(hid, shape.inter), rnd(M, hid, scale=1.0)
        fn = lambda: ops.linear_residual(a, w, h)  # noqa: E731
    elif args.kernel_case == "qkv":
        cols = (Hq + 2 * H) * D
        w, b = rnd(cols, hid), rnd(cols)
        q = torch.empty((M, Hq * D), dtype=bf, device=dev)
        kc = torch.empty((H, N, D), dtype=bf, device=dev)
        vc = torch.empty_like(kc)
        inv = shape.rope_theta ** (-torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D)
        tab = ops.rope_table(inv, 8192)
        fn = lambda: ops.qkv_rope(x, w, b, M, 0, cols, Hq, H, D, pos, tab, q_out=q, k_cache=kc, v_cache=vc)  # noqa: E731
    elif args.kernel_case == "attention":
        q = rnd(M, Hq, D, scale=1.0)
        kc, vc = rnd(H, N, D, scale=1.0), rnd(H, N, D, scale=1.0)
        out = torch.empty_like(q)
        fn = lambda: ops.attention(q, kc, vc, pos, out)  # noqa: E731
    elif args.kernel_case in ("deviation", "deviation_scores", "select"):
        # every position active (layer 1 of a blend), cached chunks with 4 sinks each and
        # a fresh query tail; enough input sets, used in turn, that none is still in L2
        # when its turn comes again (algorithmic bytes: 4 x H x D x 2 B per position)
        nbytes = 4 * N * H * D * 2
        n_sets = max(1, -(-2 * 126_000_000 // nbytes))
        sets = []
        for _ in range(n_sets):
            Kb, Vb = rnd(H, N, D, scale=1.0), rnd(H, N, D, scale=1.0)
            kf = Kb.permute(1, 0, 2).reshape(N, H * D).clone()
            vf = (Vb.permute(1, 0, 2).reshape(N, H * D).float() + 0.05 * torch.randn(
                (N, H * D), generator=g, device=dev)).to(bf)
            sets.append((kf, vf, Kb, Vb))
        act = torch.arange(N, dtype=torch.int32, device=dev)
        cached = args.chunks * args.chunk_len
        fl = torch.zeros(N, dtype=torch.uint8)
        fl[:cached] = 1
        for c in range(args.chunks):
            fl[c * args.chunk_len:c * args.chunk_len + args.n_sink] |= 2
        flags = fl.to(dev)
        budget = int(round(args.ratio * args.chunk_len))
        meta = torch.tensor([[c * args.chunk_len, args.chunk_len, budget, 0] for c in range(args.chunks)],
                            dtype=torch.int32, device=dev)
        ws = ops.SelectWorkspace(N, args.chunks, dev)
        turn = [0]

        def fn():
            kf, vf, Kb, Vb = sets[turn[0] % n_sets]
            turn[0] += 1
            if args.kernel_case == "deviation":
                ops.deviation_select(kf, vf, Kb, Vb, act, flags, meta, None, ws)
            elif args.kernel_case == "deviation_scores":  # phase 1 alone
                ops.deviation_scores(kf, vf, Kb, Vb, act, flags, ws)
            else:  # "select": phase 2 alone, from the scores already in the workspace
                ops.select_from_scores(ws.diff[:N], ws.norm[:N], flags, meta, None, ws)
        if args.kernel_case == "select":
            ops.deviation_scores(*sets[0], act, flags, ws)
        kernel_bytes = nbytes if args.kernel_case != "select" else 8 * N
    else:  # gather: 10 chunks x 512 tokens x 27 layers from the page pool
        from chunkkv_b200.store.pages import PagePool

        L = shape.n_layers
        n_pages = args.chunks * args.chunk_len // 16
        pool = PagePool(L, H, D, n_pages, dev)
        pool.pages.view(-1)[:] = 1
        table = torch.arange(n_pages, dtype=torch.int32, device=dev)
        meta = torch.tensor([[c * args.chunk_len // 16, args.chunk_len, c * args.chunk_len, 1000, 1, L, 0, 0]
                             for c in range(args.chunks)], dtype=torch.int32, device=dev)
        inv = shape.rope_theta ** (-torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D)
        kall = torch.empty((L, H, N, D), dtype=bf, device=dev)
        vall = torch.empty_like(kall)
        fn = lambda: ops.blend_gather_paged(pool.pages, table, meta, inv, kall, vall, 0, L)  # noqa: E731
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if kernel_bytes:
        # a launch of a few microseconds: time a CUDA graph of the launches (device time),
        # not the host's launch rate
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        e0.record()
        graph.replay()
        e1.record()
    else:
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    out = {"kernel_case": args.kernel_case, "ms_per_launch": ms, "shape": args.shape, "tokens": N}
    if kernel_bytes:
        pk, pk_kind = peaks()
        gbs = kernel_bytes / (ms * 1e-3) / 1e9
        out.update(bytes_per_launch=kernel_bytes, gbs=round(gbs, 1), frac_hbm=round(gbs / pk["hbm_gbs"], 4),
                   peak_source=f"{pk_kind} hbm_gbs")
    print(json.dumps(out))


def main():
    args = parse()
    if args.kernel_case:
        run_kernel_case(args)
        return
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "tp":
        run_tp(args)
    elif args.workload == "replay":
        run_replay(args)
    elif args.workload == "micro":
        run_micro(args)
    elif args.workload == "policies":
        run_policies(args)
    elif args.workload == "decode":
        run_decode(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
