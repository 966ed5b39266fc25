"""CPU oracle of the blend prefill — TEST INFRASTRUCTURE ONLY.

This module restates the reference algorithm (sarvanithin/chunkkv,
src/chunkkv/engine/torch_engine.py) with plain torch CPU ops over a
Hugging-Face-named state dict, without HF modules.  It is the checker of the
CUDA engine: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg may import it; the product path never does.

Pinning: tests/golden/make_golden.py runs the reference TorchEngine itself (on
CPU, in the container that holds the reference) and stores its outputs;
tests/test_oracle_golden.py checks this restatement against them.

One deliberate difference: the reference's pooled top-k uses an unstable
argsort (torch_engine.py:144), so the order of equal scores is undefined.  The
oracle sorts stably (equal scores: lower position first), the order the CUDA
selection kernel implements; on tie-free inputs both agree with the reference.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.nn.functional as F


@dataclass
class OracleChunk:
    """Same fields as chunkkv.engine.base.ChunkKV (base.py:13-23)."""

    keys: list
    values: list
    start: int

    @property
    def length(self) -> int:
        return self.keys[0].shape[2]


@dataclass
class OracleResult:
    logits: torch.Tensor
    logit_positions: torch.Tensor
    keys: list
    values: list
    stats: dict
    diff: torch.Tensor | None = None       # layer-1 deviation per position (fp32 [N])
    norm: torch.Tensor | None = None
    keep_abs: torch.Tensor | None = None   # positions recomputed at layers >= 1
    budget: int | None = None
    layer_times: list = field(default_factory=list)

    def chunk(self, start: int, end: int) -> OracleChunk:
        """PrefillResult.chunk (base.py:55-60): contiguous per-layer copies."""
        return OracleChunk([k[:, :, start:end, :].contiguous() for k in self.keys],
                           [v[:, :, start:end, :].contiguous() for v in self.values], start)


def plan_positions(n: int, placements, n_sink: int):
    """base.py:63-73: per-position cached / exact / sink flags."""
    cached, exact, sink = [False] * n, [False] * n, [False] * n
    for p in placements:
        for i in range(p.start, p.start + p.chunk.length):
            cached[i] = True
            if p.exact:
                exact[i] = True
            elif i < p.start + n_sink:
                sink[i] = True
    return cached, exact, sink


def py_round(x: float) -> int:
    """Python's round (half to even), as torch_engine.py:139 uses it."""
    return int(round(x))


def select(diff: torch.Tensor, norm: torch.Tensor, cached: torch.Tensor, sink: torch.Tensor,
           placements, config) -> dict[str, Any]:
    """torch_engine.py:125-147: per-chunk rel and escalation, pooled budget, top-k, keep.

    Returns keep (bool [N]), keep_abs (int64, ascending), budget (after the cap),
    chunk_stats and the eligible mask."""
    N = diff.shape[0]
    keep = (~cached) | sink
    pool = torch.zeros(N, dtype=torch.bool)
    budget = 0
    chunk_stats = []
    for p in placements:
        if p.exact:
            continue
        end = p.start + p.chunk.length
        rel = (diff[p.start:end].sum() / norm[p.start:end].sum()).item()
        ratio = config.recompute_ratio if p.ratio is None else p.ratio
        escalated = config.escalate_threshold is not None and rel > config.escalate_threshold
        if escalated:
            keep[p.start:end] = True
        elif ratio > 0:
            pool[p.start:end] = True
            budget += py_round(ratio * p.chunk.length)
        chunk_stats.append({"start": p.start, "length": p.chunk.length, "rel_dev": rel,
                            "escalated": escalated})
    eligible = pool & ~keep
    budget = min(budget, int(eligible.sum().item()))
    if budget > 0:
        scores = torch.where(eligible, diff, torch.full_like(diff, -1.0))
        top = torch.argsort(-scores, stable=True)[:budget]
        keep[top] = True
    keep_abs = keep.nonzero().squeeze(1)
    return dict(keep=keep, keep_abs=keep_abs, budget=budget, chunk_stats=chunk_stats,
                eligible=eligible)


class OracleEngine:
    """Plain restatement of TorchEngine (torch_engine.py:18-178) on CPU tensors."""

    def __init__(self, shape, state_dict: dict[str, torch.Tensor], dtype=torch.float32):
        self.shape = shape
        self.dtype = dtype
        self.n_layers = shape.n_layers
        self.n_heads, self.n_kv, self.head_dim = shape.n_heads, shape.n_kv, shape.head_dim
        self.eps = shape.rms_eps
        self.w = {k: v.to(dtype) for k, v in state_dict.items()}
        # torch_engine.py:33
        D = self.head_dim
        self.inv_freq = shape.rope_theta ** (-torch.arange(0, D, 2, dtype=torch.float32) / D)

    # -- helpers (torch_engine.py:46-76; RMSNorm and MLP as HF Qwen2 computes them)
    def _rms(self, x, w):
        x32 = x.to(torch.float32)
        var = x32.pow(2).mean(-1, keepdim=True)
        return w * (x32 * torch.rsqrt(var + self.eps)).to(x.dtype)

    def _rotate(self, x, angles):
        cos, sin = angles.cos(), angles.sin()
        half = self.head_dim // 2
        x32 = x.float()
        x1, x2 = x32[..., :half], x32[..., half:]
        return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).to(x.dtype)

    def _rope(self, x, positions):
        return self._rotate(x, positions.float()[:, None] * self.inv_freq[None, :])

    def shift_keys(self, keys, delta: int):
        if delta == 0:
            return keys
        return self._rotate(keys, (delta * self.inv_freq)[None, :].expand(keys.shape[-2], -1))

    def _lw(self, li, name):
        return self.w[f"model.layers.{li}.{name}"]

    def _qkv(self, li, x, positions):
        B, L, _ = x.shape
        q = F.linear(x, self._lw(li, "self_attn.q_proj.weight"), self._lw(li, "self_attn.q_proj.bias"))
        k = F.linear(x, self._lw(li, "self_attn.k_proj.weight"), self._lw(li, "self_attn.k_proj.bias"))
        v = F.linear(x, self._lw(li, "self_attn.v_proj.weight"), self._lw(li, "self_attn.v_proj.bias"))
        q = q.view(B, L, self.n_heads, -1).transpose(1, 2)
        k = k.view(B, L, self.n_kv, -1).transpose(1, 2)
        v = v.view(B, L, self.n_kv, -1).transpose(1, 2)
        return self._rope(q, positions), self._rope(k, positions), v

    def _attend(self, li, h, q, K, V, mask):
        out = F.scaled_dot_product_attention(q, K, V, attn_mask=mask, enable_gqa=True)
        out = out.transpose(1, 2).reshape(h.shape[0], h.shape[1], -1)
        h = h + F.linear(out, self._lw(li, "self_attn.o_proj.weight"))
        x = self._rms(h, self._lw(li, "post_attention_layernorm.weight"))
        g = F.linear(x, self._lw(li, "mlp.gate_proj.weight"))
        u = F.linear(x, self._lw(li, "mlp.up_proj.weight"))
        return h + F.linear(F.silu(g) * u, self._lw(li, "mlp.down_proj.weight"))

    def _logits(self, h):
        return F.linear(self._rms(h, self.w["model.norm.weight"]), self.w["lm_head.weight"])

    # -- torch_engine.py:80-178
    @torch.inference_mode()
    def prefill(self, tokens, placements=None, config=None, logits_from=None) -> OracleResult:
        placements = placements or []
        if config is None:
            raise ValueError("pass a BlendConfig")
        N = len(tokens)
        logits_from = N - 1 if logits_from is None else logits_from
        cached_l, exact_l, sink_l = plan_positions(N, placements, config.n_sink)
        cached = torch.tensor(cached_l)
        sink = torch.tensor(sink_l)
        fresh_idx = torch.tensor([i for i in range(N) if not cached_l[i]], dtype=torch.long)
        layer0_idx = torch.tensor([i for i in range(N) if not exact_l[i]], dtype=torch.long)
        ar = torch.arange(N)
        dt = self.dtype

        def base_kv(li):
            K = torch.zeros((1, self.n_kv, N, self.head_dim), dtype=dt)
            V = torch.zeros_like(K)
            for p in placements:
                end = p.start + p.chunk.length
                K[:, :, p.start:end] = self.shift_keys(p.chunk.keys[li].cpu().to(dt), p.start - p.chunk.start)
                V[:, :, p.start:end] = p.chunk.values[li].cpu().to(dt)
            return K, V

        emb = F.embedding(torch.tensor([tokens]), self.w["model.embed_tokens.weight"])
        active = layer0_idx if config.full_first_layer else fresh_idx
        h = emb[:, active]
        keys_out, values_out, times = [], [], []
        selected_cached = 0
        chunk_stats: list[dict] = []
        diff = norm = keep_abs = None
        budget = None
        for li in range(self.n_layers):
            t0 = time.perf_counter()
            x = self._rms(h, self._lw(li, "input_layernorm.weight"))
            q, k, v = self._qkv(li, x, active)
            K, V = base_kv(li)
            if li == 1 and placements and config.full_first_layer:
                d_act = ((k - K[:, :, active]).float() ** 2).sum(dim=(0, 1, 3))
                d_act += ((v - V[:, :, active]).float() ** 2).sum(dim=(0, 1, 3))
                n_act = (k.float() ** 2).sum(dim=(0, 1, 3)) + (v.float() ** 2).sum(dim=(0, 1, 3))
                diff = torch.zeros(N)
                norm = torch.zeros(N)
                diff[active] = d_act
                norm[active] = n_act
                sel = select(diff, norm, cached, sink, placements, config)
                chunk_stats, budget, keep_abs = sel["chunk_stats"], sel["budget"], sel["keep_abs"]
                selected_cached = int(cached[keep_abs].sum().item())
                local = torch.full((N,), -1, dtype=torch.long)
                local[active] = torch.arange(len(active))
                idx = local[keep_abs]
                assert bool((idx >= 0).all()), "selected a token that was never computed"
                h, q, k, v = h[:, idx], q[:, :, idx], k[:, :, idx], v[:, :, idx]
                active = keep_abs
            K[:, :, active] = k
            V[:, :, active] = v
            mask = active[:, None] >= ar[None, :]
            h = self._attend(li, h, q, K, V, mask)
            keys_out.append(K)
            values_out.append(V)
            times.append(time.perf_counter() - t0)
        want = (active >= logits_from).nonzero().squeeze(1)
        if len(want) != N - logits_from:
            raise ValueError("logits requested for positions that were not recomputed")
        logits = self._logits(h[:, want])[0]
        n_cached = sum(cached_l)
        layer0 = len(layer0_idx) if config.full_first_layer else N - n_cached
        rest = (N - n_cached + selected_cached) * (self.n_layers - 1)
        stats = {"tokens": N, "cached_tokens": n_cached, "recomputed_cached_tokens": selected_cached,
                 "prefill_token_equiv": (layer0 + rest) / self.n_layers, "chunks": chunk_stats}
        return OracleResult(logits, torch.arange(logits_from, N), keys_out, values_out, stats, diff,
                            norm, keep_abs, budget, times)

    def last_logprobs(self, result: OracleResult):
        """torch_engine.py:200-201."""
        return torch.log_softmax(result.logits[-1].float(), -1).numpy()
