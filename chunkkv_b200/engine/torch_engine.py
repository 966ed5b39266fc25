"""Blend prefill on B200 (drop-in for chunkkv.engine.torch_engine.TorchEngine).

Same constructor, attributes and methods as the reference
(src/chunkkv/engine/torch_engine.py:18-207); the forward runs on this
package's sm_100a kernels through the C ABI:

  plan (vectorised, host) -> one packed H2D upload of token ids, positions,
  flags and chunk tables
  K1  ckv_blend_gather_*   moved chunks -> blended cache of ALL layers, re-RoPE by
                           Delta on the fly (replaces base_kv, torch_engine.py:96-103)
  per layer:  ckv_rmsnorm -> ckv_qkv_rope (GEMM + bias + RoPE, k/v written into the
              blended cache, torch_engine.py:61-66,155-156) -> ckv_attention
              (position mask, torch_engine.py:157) -> ckv_linear_residual (o_proj)
              -> ckv_rmsnorm -> ckv_linear_swiglu -> ckv_linear_residual (down)
  layer 1:    k/v of every active token (compact) -> K2/K3 ckv_deviation_select
              (torch_engine.py:117-150) -> ckv_apply_selection -> q for the
              selected rows only -> one D2H of the selection (the only sync)
  logits:     ckv_rmsnorm + ckv_gemv / ckv_linear on the logit rows (162-165)

There is no CPU path: a missing library raises (chunkkv_b200._lib).
"""

from __future__ import annotations

import array
import math

import numpy as np
import torch

from chunkkv_b200 import _lib, ops
from chunkkv_b200.engine.base import (BlendConfig, CacheChunkKV, ChunkKV, Placement,  # noqa: F401
                                      PrefillResult, plan_arrays, plan_positions)
from chunkkv_b200.engine.staging import Staging as _Staging
from chunkkv_b200.engine.staging import pack_upload as _pack_upload
from chunkkv_b200.engine.weights import PackedQwen2, Qwen2Shape, pack


class TorchEngine:
    """Blend-prefill engine over Qwen2-family weights, running on this package's CUDA kernels."""

    def __init__(self, model, tokenizer=None, *, weights: PackedQwen2 | None = None, device=None,
                 tp=None):
        """`tp`: an `engine.tp.TensorParallel` group to split the model by KV head over
        its ranks (one process per GPU); the engine then holds and returns only this
        rank's KV heads, and `n_kv` / `layers` describe the local shard."""
        self.model = model
        self.tokenizer = tokenizer
        self.tp = tp if (tp is not None and tp.size > 1) else None
        tp_rank, tp_size = (tp.rank, tp.size) if self.tp else (0, 1)
        if weights is None:
            if model is None:
                raise ValueError("pass an HF model or packed weights")
            cfg = model.config
            scaling = getattr(cfg, "rope_scaling", None) or {}
            if scaling.get("rope_type", scaling.get("type", "default")) != "default":
                raise NotImplementedError("rope_scaling is not supported in v0")
            head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
            base = (getattr(cfg, "rope_theta", None) or scaling.get("rope_theta")
                    or cfg.rope_parameters["rope_theta"])
            shape = Qwen2Shape(
                name=getattr(cfg, "_name_or_path", "") or "qwen2", n_layers=cfg.num_hidden_layers,
                hidden=cfg.hidden_size, n_heads=cfg.num_attention_heads, n_kv=cfg.num_key_value_heads,
                head_dim=head_dim, inter=cfg.intermediate_size, vocab=cfg.vocab_size, rope_theta=float(base),
                rms_eps=float(cfg.rms_norm_eps), tied=bool(getattr(cfg, "tie_word_embeddings", False)))
            sd = dict(model.state_dict())
            if shape.tied:
                sd.setdefault("lm_head.weight", sd["model.embed_tokens.weight"])
            dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            weights = pack(shape, sd, device=dev, tp_rank=tp_rank, tp_size=tp_size)
        if (weights.tp_rank, weights.tp_size) != (tp_rank, tp_size):
            raise ValueError(f"weights are shard {weights.tp_rank}/{weights.tp_size}, "
                             f"the engine's group is rank {tp_rank} of {tp_size}")
        self.w = weights
        self.shape = s = weights.shape
        self.device = weights.device
        self.layers = getattr(getattr(model, "model", None), "layers", None) or weights.layers
        self.n_heads, self.n_kv, self.head_dim = s.n_heads, s.n_kv, s.head_dim
        D = s.head_dim
        self.inv_freq = s.rope_theta ** (-torch.arange(0, D, 2, device=self.device, dtype=torch.float32) / D)
        eos = None
        gen_cfg = getattr(model, "generation_config", None)
        if gen_cfg is not None:
            eos = gen_cfg.eos_token_id
        eos_set = set(eos if isinstance(eos, list) else ([eos] if eos is not None else []))
        tok_eos = getattr(tokenizer, "eos_token_id", None)
        self.eos = eos_set | ({tok_eos} if tok_eos is not None else set())
        self._rope_tab: torch.Tensor | None = None
        self._up = _Staging(slots=4)
        self._down = _Staging()
        self._ws: ops.SelectWorkspace | None = None
        self._attn_ws: torch.Tensor | None = None
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0
        _lib.load()  # fail loudly now if the CUDA library is missing

    @classmethod
    def load(cls, repo: str, dtype=torch.bfloat16) -> "TorchEngine":
        from transformers import AutoModelForCausalLM, AutoTokenizer

        model = AutoModelForCausalLM.from_pretrained(repo, dtype=dtype)
        return cls(model, AutoTokenizer.from_pretrained(repo))

    @classmethod
    def from_packed(cls, weights: PackedQwen2, tokenizer=None, tp=None) -> "TorchEngine":
        return cls(None, tokenizer, weights=weights, tp=tp)

    # -- helpers -----------------------------------------------------------
    def rope_table(self, n: int) -> torch.Tensor:
        if self._rope_tab is None or self._rope_tab.shape[0] < n:
            size = max(n, 4096)
            size = 1 << math.ceil(math.log2(size))
            self._rope_tab = ops.rope_table(self.inv_freq, size)
        return self._rope_tab

    def _workspace(self, n: int, n_chunks: int) -> ops.SelectWorkspace:
        ws = self._ws
        if ws is None or ws.diff.numel() < n or ws.rel.numel() < n_chunks:
            ws = self._ws = ops.SelectWorkspace(max(n, 1024), max(n_chunks, 64), self.device)
        return ws

    def _attn_workspace(self, m: int, n_ctx: int) -> torch.Tensor:
        """Scheduler words and key-split scratch of the attention kernel, zeroed once,
        grown on demand and reused."""
        s = self.shape
        need = ops.attention_workspace_bytes(m, s.n_heads, s.n_kv, s.head_dim, n_ctx)
        if self._attn_ws is None or self._attn_ws.numel() < need:
            self._attn_ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self._attn_ws

    def _fused_norm(self, m: int) -> bool:
        """Whether a decode projection of m rows can take RMSNorm(h) itself."""
        return m <= ops.GEMV_NORM_MAX_ROWS and self.shape.hidden <= ops.GEMV_NORM_MAX_K

    def shift_keys(self, keys: torch.Tensor, delta: int) -> torch.Tensor:
        """Re-RoPE post-RoPE keys (1, H, L, D) by `delta` (torch_engine.py:56-59): rotated
        in fp32 and returned in the keys' dtype (bf16 or fp32; other dtypes raise
        NotImplementedError), on this engine's device."""
        if delta == 0:
            return keys
        k = keys.to(device=self.device).contiguous()
        return ops.shift_keys(k, delta, self.inv_freq)

    def _chunk_tensors(self, chunk, li: int, kv: int) -> torch.Tensor:
        if isinstance(chunk, CacheChunkKV) and chunk.viewable:
            t = chunk.view(li, kv)[None]
            if t.device == self.device and t.dtype == torch.bfloat16:
                return t
        t = (chunk.keys if kv == 0 else chunk.values)[li]
        if not (t.is_cuda and t.dtype == torch.bfloat16 and t.stride(-1) == 1 and t.stride(-2) == t.shape[-1]
                and t.data_ptr() % 16 == 0 and t.stride(1) % 8 == 0):
            t = t.to(device=self.device, dtype=torch.bfloat16).contiguous()
        return t

    def _block_tail(self, li: int, attn, h, x, act, part, M: int, exch=None, pair: int = 0) -> bool:
        """o_proj + residual, post-attention RMSNorm, SwiGLU MLP + residual of layer `li`
        (torch_engine.py:68-76) over rows [0, M).  Tensor parallel: o_proj and down_proj
        are row-parallel, so their partial rows are summed over the ranks and the
        residual add is fused with the next RMSNorm (the next layer's input norm, or
        the final norm after the last layer); returns True when x then holds it."""
        s, lw, tp = self.shape, self.w.layers[li], self.tp
        if tp is None and M <= 8:  # decode: one warp per weight row streams the weights
            ops.gemv_residual(attn[:M], lw.w_o, h)
            if self._fused_norm(M):  # the post-attention RMSNorm inside the gate/up GEMV
                ops.gemv_swiglu(h[:M], lw.w_gu, act, norm_w=lw.ln2, eps=s.rms_eps)
            else:
                ops.rmsnorm(h[:M], lw.ln2, s.rms_eps, out=x[:M])
                ops.gemv_swiglu(x[:M], lw.w_gu, act)
            ops.gemv_residual(act[:M], lw.w_down, h)
            return False
        if tp is None:
            ops.linear_residual(attn, lw.w_o, h, m=M)
            ops.rmsnorm(h[:M], lw.ln2, s.rms_eps, out=x[:M])
            ops.linear_swiglu(x, lw.w_gu, act, m=M)
            ops.linear_residual(act, lw.w_down, h, m=M)
            return False
        nxt = self.w.layers[li + 1].ln1 if li + 1 < s.n_layers else self.w.norm
        if exch is not None:
            # partial rows read over NVLink by the owning ranks, reduced there with the
            # residual add and gathered back into every rank's h; RMSNorm locally
            for xin, wmat, norm in ((attn, lw.w_o, lw.ln2), (act, lw.w_down, nxt)):
                buf = exch.recv_toggle
                exch.recv_toggle ^= 1
                ops.linear_partial(xin[:M], wmat, exch, buf)
                ops.reduce_add_gather(exch, buf, pair, M)
                ops.rmsnorm(h[:M], norm, s.rms_eps, out=x[:M])
                if wmat is lw.w_o:
                    ops.linear_swiglu(x, lw.w_gu, act, m=M)
            return True
        ops.linear(attn[:M], lw.w_o, out=part[:M])
        tp.all_reduce_(part[:M])
        ops.add_rmsnorm(h[:M], part[:M], lw.ln2, s.rms_eps, out=x[:M])
        ops.linear_swiglu(x, lw.w_gu, act, m=M)
        ops.linear(act[:M], lw.w_down, out=part[:M])
        tp.all_reduce_(part[:M])
        ops.add_rmsnorm(h[:M], part[:M], nxt, s.rms_eps, out=x[:M])
        return True

    # -- main entry ----------------------------------------------------------
    @torch.inference_mode()
    def prefill(self, tokens, placements=None, config=None, logits_from=None) -> PrefillResult:
        from chunkkv_b200.store.pages import PagedChunkKV

        placements = placements or []
        config = config or BlendConfig()
        s = self.shape
        N = len(tokens)
        L, H, Hq, D, hid = s.n_layers, s.n_kv, s.n_heads, s.head_dim, s.hidden
        logits_from = N - 1 if logits_from is None else logits_from
        dev = self.device
        if N == 0:
            raise ValueError("empty request")

        if isinstance(tokens, list):  # the reference's list[int]: a C-level conversion
            try:
                tok_np = np.frombuffer(array.array("q", tokens), dtype=np.int64)
            except (OverflowError, TypeError):
                tok_np = np.asarray(tokens, dtype=np.int64)
        else:
            tok_np = np.asarray(tokens, dtype=np.int64)
        if tok_np.min() < 0 or tok_np.max() >= s.vocab:
            raise ValueError("token id outside the vocabulary")
        plan = plan_arrays(N, placements, config.n_sink)
        active0 = plan.layer0_idx if config.full_first_layer else plan.fresh_idx
        M0 = int(active0.size)
        do_select = bool(placements) and config.full_first_layer and L > 1

        # chunk tables for the gather: paged chunks by page list, others by tensor address
        paged_meta, dense_meta, page_table, kptr, vptr, keep_alive = [], [], [], [], [], []
        for p in placements:
            c = p.chunk
            lb = 1 if (config.full_first_layer and not p.exact) else 0
            delta = p.start - c.start
            if isinstance(c, PagedChunkKV):
                c.check_alive()
                paged_meta.append([len(page_table), c.length, p.start, delta, lb, L, c.src_offset, 0])
                page_table.extend(c.page_ids.tolist())
            else:
                ks = [self._chunk_tensors(c, li, 0) for li in range(L)]
                vs = [self._chunk_tensors(c, li, 1) for li in range(L)]
                if any(k.stride(1) != ks[0].stride(1) for k in ks + vs):
                    ks = [k.contiguous() for k in ks]
                    vs = [v.contiguous() for v in vs]
                keep_alive.append((ks, vs))
                dense_meta.append([len(kptr), c.length, p.start, delta, lb, L, 0, ks[0].stride(1)])
                kptr.extend(k.data_ptr() for k in ks)
                vptr.extend(v.data_ptr() for v in vs)

        sel_meta = []
        if do_select:
            for p in placements:
                ratio = config.recompute_ratio if p.ratio is None else p.ratio
                budget = int(round(ratio * p.chunk.length)) if ratio > 0 else -1
                sel_meta.append([p.start, p.chunk.length, budget, int(bool(p.exact))])

        parts = [("tokens", tok_np.astype(np.int32)), ("active0", active0.astype(np.int32))]
        if do_select:
            parts += [("pos_flags", plan.pos_flags()), ("sel_meta", np.asarray(sel_meta, np.int32).reshape(-1, 4))]
        if paged_meta:
            parts += [("paged_meta", np.asarray(paged_meta, np.int32)),
                      ("page_table", np.asarray(page_table, np.int32))]
        if dense_meta:
            parts += [("dense_meta", np.asarray(dense_meta, np.int32)),
                      ("kptr", np.asarray(kptr, np.uint64)), ("vptr", np.asarray(vptr, np.uint64))]
        d, h2d = _pack_upload(parts, self._up, dev)
        self.last_h2d_bytes = h2d

        rope_tab = self.rope_table(N)
        # algorithmic work of the bandwidth / attention kernels (roofline accounting only)
        kv_row = 2 * H * D * 2  # K+V bytes of one token in one layer
        gather_bytes = 2.0 * kv_row * sum(
            p.chunk.length * (L - (1 if (config.full_first_layer and not p.exact) else 0)) for p in placements)
        attn_flops = 4.0 * Hq * D * float((active0.astype(np.int64) + 1).sum())
        bf = dict(dtype=torch.bfloat16, device=dev)
        K_all = torch.empty((L, H, N, D), **bf)
        V_all = torch.empty((L, H, N, D), **bf)
        if paged_meta:
            pools = {id(p.chunk.pool): p.chunk.pool for p in placements if isinstance(p.chunk, PagedChunkKV)}
            if len(pools) != 1:
                raise ValueError("paged chunks of one request must come from one page pool")
            pool = next(iter(pools.values()))
            ops.blend_gather_paged(pool.pages, d["page_table"], d["paged_meta"], self.inv_freq, K_all, V_all, 0, L,
                                   nbytes=gather_bytes * len(paged_meta) / len(placements))
        if dense_meta:
            ops.blend_gather_dense(d["kptr"], d["vptr"], d["dense_meta"], self.inv_freq, K_all, V_all, 0, L,
                                   nbytes=gather_bytes * len(dense_meta) / len(placements))

        tp = self.tp
        exch = tp.exchange(max(M0, 1), hid, dev) if (tp and tp.fused) else None
        pair = 0  # h / x pair of the exchange in use (the selection moves to the other)
        if exch is not None:
            h, x = exch.h[0][:max(M0, 1)], exch.x[0][:max(M0, 1)]
        else:
            h = torch.empty((max(M0, 1), hid), **bf)
            x = torch.empty_like(h)
        q = torch.empty((max(M0, 1), Hq * D), **bf)
        attn = torch.empty_like(q)
        act = torch.empty((max(M0, 1), s.inter), **bf)
        part = torch.empty_like(h) if (tp and exch is None) else None  # partial rows for NCCL
        x_ready = False  # x already holds RMSNorm(h) for this layer (fused into the last add)
        if M0:
            ops.embed(self.w.embed, d["tokens"], d["active0"], h[:M0])
        active = d["active0"]
        M = M0
        active_host = active0
        selected_cached = 0
        chunk_stats: list[dict] = []
        ws = None
        qkv_cols = (Hq + 2 * H) * D
        for li in range(L):
            lw = self.w.layers[li]
            if M == 0:
                break
            if not x_ready:
                ops.rmsnorm(h[:M], lw.ln1, s.rms_eps, out=x[:M])
            x_ready = False
            if li == 1 and do_select:
                ws = self._workspace(N, len(placements))
                kc = torch.empty((M, H * D), **bf)
                vc = torch.empty((M, H * D), **bf)
                ops.qkv_rope(x, lw.w_qkv, lw.b_qkv, M, Hq * D, qkv_cols, Hq, H, D, active, rope_tab,
                             k_compact=kc, v_compact=vc)
                if tp:
                    # each rank scores its own KV heads; the sum over ranks is the
                    # reference's sum over all heads (torch_engine.py:118-124)
                    ops.deviation_scores(kc, vc, K_all[1], V_all[1], active, d["pos_flags"], ws)
                    tp.all_reduce_(ws.scores)
                    ops.select_from_scores(ws.diff, ws.norm, d["pos_flags"], d["sel_meta"],
                                           config.escalate_threshold, ws)
                else:
                    ops.deviation_select(kc, vc, K_all[1], V_all[1], active, d["pos_flags"], d["sel_meta"],
                                         config.escalate_threshold, ws)
                if exch is not None:
                    h2, x2 = exch.h[1 - pair][:h.shape[0]], exch.x[1 - pair][:x.shape[0]]
                    pair = 1 - pair
                else:
                    h2, x2 = torch.empty_like(h), torch.empty_like(x)
                ops.apply_selection(ws, M, h, h2, x, x2, kc, vc, K_all[1], V_all[1])
                # the one host sync: selection size, chunk deviations, kept positions
                n_ch = len(placements)
                down = self._down.get(4 * (8 + n_ch + N))
                hv = down.view(torch.int32)
                hv[:8].copy_(ws.counts, non_blocking=True)
                hv[8:8 + n_ch].copy_(ws.rel[:n_ch].view(torch.int32), non_blocking=True)
                hv[8 + n_ch:8 + n_ch + N].copy_(ws.keep_abs[:N], non_blocking=True)
                torch.cuda.current_stream().synchronize()
                counts = hv[:8].numpy().copy()
                rel = hv[8:8 + n_ch].view(torch.float32).numpy().astype(np.float64)
                if counts[5] & 0x1:  # CKV_DEV_ERR_WAIT_TIMEOUT: a bounded device wait ran out
                    raise RuntimeError("layer-1 selection: a device wait ran out (see ckv_get_device_error)")
                if counts[5]:
                    raise AssertionError("selected a token that was never computed")
                M = int(counts[0])
                selected_cached = int(counts[1])
                h, x = h2, x2
                active = ws.keep_abs[:M]
                # the GPU waits on this host: launch the next kernel first, then the bookkeeping
                if M:
                    ops.qkv_rope(x, lw.w_qkv, lw.b_qkv, M, 0, Hq * D, Hq, H, D, active, rope_tab, q_out=q)
                active_host = hv[8 + n_ch:8 + n_ch + M].numpy().copy()
                self.last_d2h_bytes = 4 * (8 + n_ch + N)
                thr = config.escalate_threshold
                for p, r in zip(placements, rel):
                    if p.exact:
                        continue
                    chunk_stats.append({"start": p.start, "length": p.chunk.length, "rel_dev": float(r),
                                        "escalated": thr is not None and float(r) > thr})
                attn_flops = 4.0 * Hq * D * float((active_host.astype(np.int64) + 1).sum())
            else:
                ops.qkv_rope(x, lw.w_qkv, lw.b_qkv, M, 0, qkv_cols, Hq, H, D, active, rope_tab, q_out=q,
                             k_cache=K_all[li], v_cache=V_all[li])
            if M == 0:
                break
            ops.attention(q, K_all[li], V_all[li], active, attn, m=M, flops=attn_flops,
                          workspace=self._attn_workspace(M, N))
            x_ready = self._block_tail(li, attn, h, x, act, part, M, exch, pair)

        r0 = int(np.searchsorted(active_host, logits_from, side="left"))
        n_log = M - r0
        if n_log != N - logits_from:
            raise ValueError("logits requested for positions that were not recomputed")
        if n_log > 0:
            # after the last layer a tensor-parallel run already holds norm(h) in x
            xf = x[r0:M] if (x_ready and li == L - 1) else ops.rmsnorm(h[r0:M], self.w.norm, s.rms_eps)
            logits = ops.gemv(xf, self.w.lm_head) if n_log <= 8 else ops.linear(xf, self.w.lm_head)
        else:
            logits = torch.empty((0, s.vocab), **bf)

        n_cached = int(plan.cached.sum())
        layer0 = M0 if config.full_first_layer else N - n_cached
        if not do_select:
            selected_cached = 0
        rest = (N - n_cached + selected_cached) * (L - 1)
        stats = {"tokens": N, "cached_tokens": n_cached, "recomputed_cached_tokens": selected_cached,
                 "prefill_token_equiv": (layer0 + rest) / L, "chunks": chunk_stats}
        keys = [K_all[li].unsqueeze(0) for li in range(L)]
        values = [V_all[li].unsqueeze(0) for li in range(L)]
        del keep_alive
        return PrefillResult(logits, torch.arange(logits_from, N), keys, values, stats,
                             copy=lambda t: t.contiguous(), cache=(K_all, V_all), selected=active.clone())

    # -- decode ----------------------------------------------------------------
    @torch.inference_mode()
    def generate(self, result: PrefillResult, max_tokens: int = 32) -> list[int]:
        """Greedy decode continuing a prefill (torch_engine.py:180-198), on the same kernels:
        the cache is sized once for the new tokens instead of a torch.cat per step.  The
        projections are the m = 1 GEMV kernels; the next token and the position stay on
        the device, and after the first step one decode step is replayed as a CUDA graph
        (one-GPU engines), so the host only reads back each token id."""
        s = self.shape
        L, H, Hq, D, hid = s.n_layers, s.n_kv, s.n_heads, s.head_dim, s.hidden
        dev = self.device
        K0, V0 = result.cache if result.cache is not None else (
            torch.cat(list(result.keys), 0), torch.cat(list(result.values), 0))
        pos = K0.shape[2]
        cap = pos + max(1, max_tokens)
        K = torch.zeros((L, H, cap, D), dtype=torch.bfloat16, device=dev)
        V = torch.zeros_like(K)
        K[:, :, :pos].copy_(K0)
        V[:, :, :pos].copy_(V0)
        out: list[int] = []
        nxt = int(result.logits[-1].float().argmax().item())
        bf = dict(dtype=torch.bfloat16, device=dev)
        exch = self.tp.exchange(1, hid, dev) if (self.tp and self.tp.fused) else None
        if exch is not None:
            h, x = exch.h[0][:1], exch.x[0][:1]
        else:
            h = torch.empty((1, hid), **bf)
            x = torch.empty_like(h)
        q = torch.empty((1, Hq * D), **bf)
        attn = torch.empty_like(q)
        act = torch.empty((1, s.inter), **bf)
        xf = torch.empty_like(h)
        logits = torch.empty((1, s.vocab), **bf)
        part = torch.empty_like(h) if (self.tp and exch is None) else None
        tok = torch.full((1,), nxt, dtype=torch.int32, device=dev)
        posd = torch.full((1,), pos, dtype=torch.int32, device=dev)
        rope_tab = self.rope_table(cap)
        attn_ws = self._attn_workspace(1, cap)

        def step():  # token tok at position posd -> next token in tok, posd + 1
            ops.embed(self.w.embed, tok, None, h)
            x_ready = False
            for li in range(L):
                lw = self.w.layers[li]
                # q, and k / v into this layer's cache [H, cap, D] at position posd
                if not x_ready and self._fused_norm(1):  # the input RMSNorm inside the QKV GEMV
                    ops.gemv_qkv_rope(h, lw.w_qkv, lw.b_qkv, Hq, H, D, posd, rope_tab, q, K[li], V[li],
                                      norm_w=lw.ln1, eps=s.rms_eps)
                else:
                    if not x_ready:
                        ops.rmsnorm(h, lw.ln1, s.rms_eps, out=x)
                    ops.gemv_qkv_rope(x, lw.w_qkv, lw.b_qkv, Hq, H, D, posd, rope_tab, q, K[li], V[li])
                ops.attention(q, K[li], V[li], posd, attn, m=1, workspace=attn_ws)
                x_ready = self._block_tail(li, attn, h, x, act, part, 1, exch, 0)
            last = x if x_ready else ops.rmsnorm(h, self.w.norm, s.rms_eps, out=xf)
            ops.gemv(last, self.w.lm_head, out=logits)
            ops.greedy_next(logits[0], tok, posd)  # argmax into tok, posd += 1

        graph = None
        use_graph = self.tp is None and ops._TIMER is None
        while len(out) < max_tokens and nxt not in self.eos:
            out.append(nxt)
            if graph is not None:
                graph.replay()
            else:
                step()
                if use_graph and len(out) < max_tokens:
                    try:
                        g = torch.cuda.CUDAGraph()
                        with torch.cuda.graph(g):
                            step()
                        graph = g
                    except RuntimeError:
                        use_graph = False  # capture refused: keep stepping eagerly
            nxt = int(tok.item())
        return out

    def last_logprobs(self, result: PrefillResult) -> np.ndarray:
        """log_softmax of the last logit row, on the device, copied to the host."""
        row = result.logits[-1].contiguous()
        return ops.log_softmax(row).cpu().numpy()

    def sync(self) -> None:
        torch.cuda.synchronize()

    def clear_cache(self) -> None:
        torch.cuda.empty_cache()
