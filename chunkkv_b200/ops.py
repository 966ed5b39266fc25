"""Torch-tensor front end of the C ABI: shape/dtype/device checks, then one call.

Every op runs on the current CUDA stream and launches the library's own
kernels; nothing here computes on the host.  Tensors are bf16 unless noted.
"""

from __future__ import annotations

import math

import torch

from chunkkv_b200 import _lib

BF16 = torch.bfloat16
PAGE_TOKENS = 16
META_STRIDE = 8
SEL_META_STRIDE = 4
SELECT_CONTROL_BYTES = 8448  # CKV_SELECT_CONTROL_BYTES: ticket + first-level histogram


def select_scratch_bytes(n_ctx: int) -> int:
    """CKV_SELECT_SCRATCH_BYTES: a score key and a flag byte per position (rounded to 16)."""
    return 5 * ((n_ctx + 15) // 16 * 16)


class LaunchTimer:
    """Records a CUDA-event pair around every kernel launch made through this module
    while installed (``with LaunchTimer() as t: ...``), with the launch's algorithmic
    work (FLOPs and HBM bytes) for roofline accounting."""

    def __init__(self, gate_us: float = 0.0):
        self.records: list[tuple[str, float, float, torch.cuda.Event, torch.cuda.Event]] = []
        self.kernels: dict[str, int] = {}  # device kernels launched per entry point
        # With gate_us > 0 the stream first runs a device sleep of about gate_us (SM cycles
        # counted at the top clock, so longer at lower clocks) before each timed launch: the
        # launch is queued behind it, and its event pair then measures the kernel rather
        # than the host's time to submit it.
        self.gate_cycles = int(gate_us * 1965)

    def __enter__(self):
        global _TIMER
        self._prev, _TIMER = _TIMER, self
        return self

    def __exit__(self, *exc):
        global _TIMER
        _TIMER = self._prev
        return False

    def summary(self) -> dict[str, dict]:
        """Per entry point: launches, total ms, FLOPs and bytes (events must have completed)."""
        out: dict[str, dict] = {}
        for name, flops, nbytes, e0, e1 in self.records:
            d = out.setdefault(name, {"launches": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0})
            d["launches"] += 1
            d["ms"] += e0.elapsed_time(e1)
            d["flops"] += flops
            d["bytes"] += nbytes
        for name, d in out.items():
            d["kernels"] = self.kernels.get(name, d["launches"])
        return out


_TIMER: LaunchTimer | None = None


def _run(name: str, *args, flops: float = 0.0, nbytes: float = 0.0, kernels: int = 1) -> None:
    t = _TIMER
    if t is None:
        _lib.call(name, *args)
        return
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if t.gate_cycles:
        torch.cuda._sleep(t.gate_cycles)
    e0.record()
    _lib.call(name, *args)
    e1.record()
    t.records.append((name, float(flops), float(nbytes), e0, e1))
    t.kernels[name] = t.kernels.get(name, 0) + kernels


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("chunkkv_b200 ops take CUDA tensors (there is no CPU path)")


def _bf16(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and t.dtype != BF16:
            raise ValueError(f"expected bfloat16, got {t.dtype}")


def _contig(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_contiguous():
            raise ValueError("expected a contiguous tensor")


def _buf(name: str, t: torch.Tensor, numel: int, dtype: torch.dtype = BF16, cols: int | None = None) -> None:
    """`t` is a contiguous `dtype` tensor of at least `numel` elements (with a last
    dimension of `cols`, when given): the kernels index it as a dense row-major array."""
    if t.dtype != dtype:
        raise ValueError(f"{name}: expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous tensor")
    if cols is not None and (t.dim() == 0 or t.shape[-1] != cols):
        raise ValueError(f"{name}: expected rows of {cols} elements, got shape {tuple(t.shape)}")
    if t.numel() < numel:
        raise ValueError(f"{name}: has {t.numel()} elements, needs at least {numel}")


def _weight(name: str, w: torch.Tensor, n: int | None, k: int) -> int:
    """`w` is a contiguous bf16 [n][k] matrix (any n when `n` is None); returns n."""
    if w.dim() != 2 or w.shape[1] != k or (n is not None and w.shape[0] != n):
        raise ValueError(f"{name}: expected shape ({'n' if n is None else n}, {k}), got {tuple(w.shape)}")
    _buf(name, w, 0)
    return w.shape[0]


def _cache(name: str, c: torch.Tensor, heads: int, head_dim: int) -> None:
    """One layer's K or V cache: contiguous bf16 [heads, n_ctx, head_dim]."""
    if c.dim() != 3 or c.shape[0] != heads or c.shape[2] != head_dim:
        raise ValueError(f"{name}: expected shape ({heads}, n_ctx, {head_dim}), got {tuple(c.shape)}")
    _buf(name, c, 0)


def _rope_tab(tab: torch.Tensor, head_dim: int) -> None:
    """A table from ``rope_table``: contiguous float32 [max_pos, head_dim / 2, 2]."""
    if tab.dim() != 3 or tab.shape[1] * 2 != head_dim or tab.shape[2] != 2:
        raise ValueError(f"rope_tab: expected shape (max_pos, {head_dim // 2}, 2), got {tuple(tab.shape)}")
    _buf("rope_tab", tab, 0, dtype=torch.float32)


def _rows_k(x: torch.Tensor) -> tuple[int, int]:
    """The (rows, k) of a contiguous bf16 [m, k] GEMV input."""
    if x.dim() != 2:
        raise ValueError(f"x: expected an [m, k] matrix, got shape {tuple(x.shape)}")
    _buf("x", x, 0)
    return x.shape[0], x.shape[1]


def _pool(pool: torch.Tensor) -> tuple[int, int, int, int]:
    """A page pool [n_pages][n_layers][2][H][PAGE_TOKENS][D]: returns (n_pages, n_layers, H, D)."""
    if pool.dim() != 6 or pool.shape[2] != 2 or pool.shape[4] != PAGE_TOKENS:
        raise ValueError(f"pool: expected shape (pages, layers, 2, H, {PAGE_TOKENS}, D), got {tuple(pool.shape)}")
    _buf("pool", pool, 0)
    return pool.shape[0], pool.shape[1], pool.shape[3], pool.shape[5]


def _table(name: str, t: torch.Tensor, stride: int) -> int:
    """An int32 [rows][stride] metadata table: returns rows."""
    if t.dim() != 2 or t.shape[1] != stride:
        raise ValueError(f"{name}: expected shape (rows, {stride}), got {tuple(t.shape)}")
    _buf(name, t, 0, dtype=torch.int32)
    return t.shape[0]


def _addresses(name: str, t: torch.Tensor, n: int) -> None:
    """A device array of at least `n` 64-bit device addresses."""
    if t.element_size() != 8 or t.is_floating_point():
        raise ValueError(f"{name}: expected 64-bit integer addresses, got {t.dtype}")
    _buf(name, t, n, dtype=t.dtype)


def _gather_out(k_out: torch.Tensor, v_out: torch.Tensor, H: int, D: int, layer_lo: int, layer_hi: int) -> None:
    """Blended caches [>= layer_hi - layer_lo][H][n_ctx][D], both of one shape."""
    for name, t in (("k_out", k_out), ("v_out", v_out)):
        if t.dim() != 4 or t.shape[1] != H or t.shape[3] != D or t.shape[0] < layer_hi - layer_lo:
            raise ValueError(f"{name}: expected shape (>= {layer_hi - layer_lo}, {H}, n_ctx, {D}), "
                             f"got {tuple(t.shape)}")
        _buf(name, t, 0)
    if k_out.shape != v_out.shape:
        raise ValueError("k_out and v_out differ in shape")
    if not 0 <= layer_lo <= layer_hi:
        raise ValueError(f"layer range [{layer_lo}, {layer_hi}) is empty or negative")


def _fresh_rows(k_fresh: torch.Tensor, v_fresh: torch.Tensor, rows: int, H: int, D: int) -> None:
    """Fresh k/v rows [>= rows][>= H*D] with unit column stride and one common row stride."""
    for name, t in (("k_fresh", k_fresh), ("v_fresh", v_fresh)):
        if t.dtype != BF16:
            raise ValueError(f"{name}: expected {BF16}, got {t.dtype}")
        if t.dim() != 2 or t.stride(1) != 1 or t.shape[1] < H * D or t.shape[0] < rows:
            raise ValueError(f"{name}: expected rows of {H * D} contiguous elements (at least {rows} rows), "
                             f"got shape {tuple(t.shape)} with strides {t.stride()}")
    if k_fresh.stride(0) != v_fresh.stride(0):
        raise ValueError("k_fresh and v_fresh differ in row stride")


def _select_ws(ws: "SelectWorkspace", n_ctx: int, n_chunks: int) -> None:
    if ws.keep_abs.numel() < n_ctx or ws.diff.numel() < n_ctx or ws.scratch.numel() < select_scratch_bytes(n_ctx) or ws.rel.numel() < n_chunks:
        raise ValueError(f"selection workspace too small for {n_ctx} positions and {n_chunks} chunks")


# ------------------------------------------------------------------ re-RoPE
def rope_table(inv_freq: torch.Tensor, max_pos: int) -> torch.Tensor:
    """(cos, sin) of fp32(p * inv_freq[j]) for p < max_pos: float32 [max_pos, half, 2]."""
    _cuda(inv_freq)
    half = inv_freq.numel()
    out = torch.empty((max_pos, half, 2), dtype=torch.float32, device=inv_freq.device)
    _run("ckv_rope_table", _ptr(inv_freq), half, max_pos, _ptr(out), _stream())
    return out


# rotation entry point per key dtype: the reference rotates in fp32 and returns the
# input dtype (torch_engine.py:46-51), so bf16 keys come back bf16 and fp32 keys fp32
_ROPE_DTYPES = {torch.bfloat16: "", torch.float32: "_f32"}


def _rope_suffix(t: torch.Tensor, what: str) -> str:
    if t.dtype not in _ROPE_DTYPES:
        raise NotImplementedError(f"{what}: dtype {t.dtype} is not supported (bfloat16 and float32 are)")
    return _ROPE_DTYPES[t.dtype]


def shift_keys(keys: torch.Tensor, delta: int, inv_freq: torch.Tensor, rot_dims: int | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Rotate post-RoPE keys (..., L, D) by `delta` positions (new tensor unless `out`),
    in fp32, returned in the keys' dtype (bf16 or fp32)."""
    sfx = _rope_suffix(keys, "shift_keys")
    _cuda(keys, inv_freq)
    _contig(keys)
    D = keys.shape[-1]
    rot = D if rot_dims is None else rot_dims
    out = torch.empty_like(keys) if out is None else out
    if out.dtype != keys.dtype or out.shape != keys.shape or not out.is_contiguous():
        raise ValueError("shift_keys: out must be a contiguous tensor of the keys' shape and dtype")
    _run("ckv_shift_keys" + sfx, _ptr(keys), _ptr(out), keys.numel() // D, D, rot, int(delta),
         _ptr(inv_freq), _stream())
    return out


def apply_rope(x: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor,
               rot_dims: int | None = None) -> torch.Tensor:
    """RoPE of x (..., L, D) at int positions (L,), in fp32, returned in x's dtype
    (bf16 or fp32)."""
    sfx = _rope_suffix(x, "apply_rope")
    _cuda(x, positions, inv_freq)
    _contig(x)
    D, L = x.shape[-1], x.shape[-2]
    pos = positions.to(torch.int32).contiguous()
    if pos.numel() != L:
        raise ValueError(f"positions has {pos.numel()} entries for sequence length {L}")
    out = torch.empty_like(x)
    rot = D if rot_dims is None else rot_dims
    _run("ckv_apply_rope" + sfx, _ptr(x), _ptr(out), x.numel() // (D * L) if L else 0, L, D, rot,
         _ptr(pos), _ptr(inv_freq), _stream())
    return out


# ---------------------------------------------------------- gather / scatter
def blend_gather_paged(pool: torch.Tensor, page_table: torch.Tensor, chunk_meta: torch.Tensor,
                       inv_freq: torch.Tensor, k_out: torch.Tensor, v_out: torch.Tensor,
                       layer_lo: int, layer_hi: int, rot_dims: int | None = None,
                       nbytes: float = 0.0) -> None:
    """Moved cached chunks (paged) -> blended cache k_out/v_out [layers, H, N, D]."""
    n_pages, n_layers, H, D = _pool(pool)
    _buf("page_table", page_table, 0, dtype=torch.int32)
    _table("chunk_meta", chunk_meta, META_STRIDE)
    _buf("inv_freq", inv_freq, (D if rot_dims is None else rot_dims) // 2, dtype=torch.float32)
    _gather_out(k_out, v_out, H, D, layer_lo, layer_hi)
    if layer_hi > n_layers:
        raise ValueError(f"layer range [{layer_lo}, {layer_hi}) past the pool's {n_layers} layers")
    _cuda(pool, page_table, chunk_meta, inv_freq, k_out, v_out)
    _run("ckv_blend_gather_paged", _ptr(pool), n_pages, _ptr(page_table), _ptr(chunk_meta),
              chunk_meta.shape[0], _ptr(inv_freq), D if rot_dims is None else rot_dims, _ptr(k_out),
              _ptr(v_out), layer_lo, layer_hi, n_layers, H, D, k_out.shape[2], _stream(), nbytes=nbytes)


def blend_gather_dense(k_ptrs: torch.Tensor, v_ptrs: torch.Tensor, chunk_meta: torch.Tensor,
                       inv_freq: torch.Tensor, k_out: torch.Tensor, v_out: torch.Tensor,
                       layer_lo: int, layer_hi: int, rot_dims: int | None = None,
                       nbytes: float = 0.0) -> None:
    """Moved cached chunks (per-layer tensors, by address) -> blended cache."""
    if k_out.dim() != 4:
        raise ValueError(f"k_out: expected shape (layers, H, n_ctx, D), got {tuple(k_out.shape)}")
    H, D = k_out.shape[1], k_out.shape[3]
    _gather_out(k_out, v_out, H, D, layer_lo, layer_hi)
    _table("chunk_meta", chunk_meta, META_STRIDE)
    _addresses("k_ptrs", k_ptrs, 0)
    _addresses("v_ptrs", v_ptrs, k_ptrs.numel())
    _buf("inv_freq", inv_freq, (D if rot_dims is None else rot_dims) // 2, dtype=torch.float32)
    _cuda(k_ptrs, v_ptrs, chunk_meta, inv_freq, k_out, v_out)
    _run("ckv_blend_gather_dense", _ptr(k_ptrs), _ptr(v_ptrs), _ptr(chunk_meta),
              chunk_meta.shape[0], _ptr(inv_freq), D if rot_dims is None else rot_dims, _ptr(k_out),
              _ptr(v_out), layer_lo, layer_hi, H, D, k_out.shape[2], _stream(), nbytes=nbytes)


def pages_write(pool: torch.Tensor, page_ids: torch.Tensor, length: int, k_ptrs: torch.Tensor,
                v_ptrs: torch.Tensor, head_stride: int) -> None:
    """`length` tokens of every layer's (H, >= length, D) sources, by address, into the
    pages page_ids[0 .. ceil(length / 16))."""
    n_pages, n_layers, H, D = _pool(pool)
    _buf("page_ids", page_ids, -(-length // PAGE_TOKENS), dtype=torch.int32)
    _addresses("k_ptrs", k_ptrs, n_layers)
    _addresses("v_ptrs", v_ptrs, n_layers)
    _cuda(pool, page_ids, k_ptrs, v_ptrs)
    _run("ckv_pages_write", _ptr(pool), n_pages, _ptr(page_ids), length, _ptr(k_ptrs),
              _ptr(v_ptrs), head_stride, n_layers, H, D, _stream())


# ------------------------------------------------------ deviation / selection
def deviation_select(k_fresh: torch.Tensor, v_fresh: torch.Tensor, k_base: torch.Tensor,
                     v_base: torch.Tensor, active: torch.Tensor, pos_flags: torch.Tensor,
                     sel_meta: torch.Tensor, threshold: float | None, ws: "SelectWorkspace") -> None:
    """Layer-1 deviation + pooled top-k into the workspace (no host sync)."""
    if k_base.dim() != 3:
        raise ValueError(f"k_base: expected shape (H, n_ctx, D), got {tuple(k_base.shape)}")
    H, n_ctx, D = k_base.shape
    _cache("k_base", k_base, H, D)
    _cache("v_base", v_base, H, D)
    _buf("active", active, 0, dtype=torch.int32)
    _fresh_rows(k_fresh, v_fresh, active.numel(), H, D)
    _buf("pos_flags", pos_flags, n_ctx, dtype=torch.uint8)
    _select_ws(ws, n_ctx, _table("sel_meta", sel_meta, SEL_META_STRIDE))
    _cuda(k_fresh, v_fresh, k_base, v_base, active, pos_flags, sel_meta)
    _run("ckv_deviation_select", _ptr(k_fresh), _ptr(v_fresh), k_fresh.stride(0), _ptr(k_base),
              _ptr(v_base), _ptr(active), active.numel(), _ptr(pos_flags), n_ctx, _ptr(sel_meta),
              sel_meta.shape[0], int(threshold is not None), float(threshold or 0.0), H, D,
              _ptr(ws.diff), _ptr(ws.norm), _ptr(ws.rel), _ptr(ws.keep_abs), _ptr(ws.sel),
              _ptr(ws.counts), _ptr(ws.scratch), _ptr(ws.control), _stream())


def deviation_scores(k_fresh: torch.Tensor, v_fresh: torch.Tensor, k_base: torch.Tensor,
                     v_base: torch.Tensor, active: torch.Tensor, pos_flags: torch.Tensor,
                     ws: "SelectWorkspace") -> None:
    """Layer-1 diff/norm of the given KV heads into ws.diff / ws.norm (no selection)."""
    if k_base.dim() != 3:
        raise ValueError(f"k_base: expected shape (H, n_ctx, D), got {tuple(k_base.shape)}")
    H, n_ctx, D = k_base.shape
    _cache("k_base", k_base, H, D)
    _cache("v_base", v_base, H, D)
    _buf("active", active, 0, dtype=torch.int32)
    _fresh_rows(k_fresh, v_fresh, active.numel(), H, D)
    _buf("pos_flags", pos_flags, n_ctx, dtype=torch.uint8)
    _select_ws(ws, n_ctx, 0)
    _cuda(k_fresh, v_fresh, k_base, v_base, active, pos_flags)
    _run("ckv_deviation_scores", _ptr(k_fresh), _ptr(v_fresh), k_fresh.stride(0), _ptr(k_base),
         _ptr(v_base), _ptr(active), active.numel(), _ptr(pos_flags), n_ctx, H, D, _ptr(ws.diff),
         _ptr(ws.norm), _stream())


def select_from_scores(diff: torch.Tensor, norm: torch.Tensor, pos_flags: torch.Tensor,
                       sel_meta: torch.Tensor, threshold: float | None,
                       ws: "SelectWorkspace") -> None:
    """The pooled selection from summed fp32 scores diff/norm [n_ctx] (every non-exact
    position active), into the workspace."""
    n_ctx = pos_flags.numel()
    _buf("pos_flags", pos_flags, n_ctx, dtype=torch.uint8)
    _buf("diff", diff, n_ctx, dtype=torch.float32)
    _buf("norm", norm, n_ctx, dtype=torch.float32)
    _select_ws(ws, n_ctx, _table("sel_meta", sel_meta, SEL_META_STRIDE))
    _cuda(diff, norm, pos_flags, sel_meta)
    _run("ckv_select_from_scores", _ptr(diff), _ptr(norm), _ptr(pos_flags), pos_flags.numel(),
              _ptr(sel_meta), sel_meta.shape[0], int(threshold is not None), float(threshold or 0.0),
              _ptr(ws.rel), _ptr(ws.keep_abs), _ptr(ws.sel), _ptr(ws.counts), _ptr(ws.scratch),
              _stream())


class SelectWorkspace:
    """Device buffers of one selection (sized for n_ctx positions, n_chunks chunks)."""

    def __init__(self, n_ctx: int, n_chunks: int, device):
        f32 = dict(dtype=torch.float32, device=device)
        i32 = dict(dtype=torch.int32, device=device)
        self.scores = torch.zeros((2, n_ctx), **f32)  # one buffer, so ranks can sum both at once
        self.diff = self.scores[0]
        self.norm = self.scores[1]
        self.rel = torch.zeros(max(1, n_chunks), **f32)
        self.keep_abs = torch.empty(n_ctx, **i32)
        self.sel = torch.empty(n_ctx, **i32)
        self.counts = torch.zeros(8, **i32)
        # per position: a 4-byte score key and a flag byte (used by the selection when
        # n_ctx is larger than what it keeps in shared memory)
        self.scratch = torch.zeros(select_scratch_bytes(n_ctx), dtype=torch.uint8, device=device)
        # ticket counter and first-level histogram: zero now, left zero by every launch
        self.control = torch.zeros(SELECT_CONTROL_BYTES // 4, **i32)


def apply_selection(ws: SelectWorkspace, max_rows: int, h_in, h_out, x_in, x_out, k_fresh, v_fresh,
                    k_cache, v_cache) -> None:
    """Rows sel[:counts[0]] of h_in/x_in -> h_out/x_out, and their fresh k/v into the
    caches at keep_abs (at most `max_rows` rows)."""
    if k_cache.dim() != 3:
        raise ValueError(f"k_cache: expected shape (H, n_ctx, D), got {tuple(k_cache.shape)}")
    H, n_ctx, D = k_cache.shape
    _cache("k_cache", k_cache, H, D)
    _cache("v_cache", v_cache, H, D)
    hidden = h_in.shape[-1]
    for name, t in (("h_in", h_in), ("h_out", h_out), ("x_in", x_in), ("x_out", x_out)):
        _buf(name, t, max_rows * hidden, cols=hidden)
    _fresh_rows(k_fresh, v_fresh, max_rows, H, D)
    _select_ws(ws, n_ctx, 0)
    _cuda(h_in, h_out, x_in, x_out, k_fresh, v_fresh, k_cache, v_cache)
    _run("ckv_apply_selection", _ptr(ws.sel), _ptr(ws.keep_abs), _ptr(ws.counts), max_rows,
              _ptr(h_in), _ptr(h_out), _ptr(x_in), _ptr(x_out), h_in.shape[-1], _ptr(k_fresh),
              _ptr(v_fresh), k_fresh.stride(0), _ptr(k_cache), _ptr(v_cache), H, D, n_ctx, _stream())


# ------------------------------------------------------------ decoder pieces
def embed(table: torch.Tensor, tokens: torch.Tensor, rows: torch.Tensor | None,
          out: torch.Tensor) -> torch.Tensor:
    n = out.shape[0]
    if table.dim() != 2:
        raise ValueError(f"table: expected a [vocab, hidden] matrix, got shape {tuple(table.shape)}")
    _buf("table", table, 0)
    _buf("out", out, n * table.shape[1], cols=table.shape[1])
    _buf("tokens", tokens, 0 if rows is not None else n, dtype=torch.int32)
    if rows is not None:
        _buf("rows", rows, n, dtype=torch.int32)
    _cuda(table, tokens, rows, out)
    _run("ckv_embed", _ptr(table), table.shape[0], table.shape[1], _ptr(tokens), _ptr(rows), n,
              _ptr(out), _stream())
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    hidden = x.shape[-1]
    rows = x.numel() // hidden if hidden else 0
    _buf("x", x, 0)
    _buf("w", w, hidden)
    if out is not None:
        _buf("out", out, rows * hidden, cols=hidden)
    _cuda(x, w, out)
    out = torch.empty_like(x) if out is None else out
    _run("ckv_rmsnorm", _ptr(x), _ptr(w), _ptr(out), rows, x.shape[-1], float(eps), _stream())
    return out


def add_rmsnorm(h: torch.Tensor, delta: torch.Tensor, w: torch.Tensor, eps: float,
                out: torch.Tensor) -> torch.Tensor:
    """h = bf16(h + delta) in place, then out = RMSNorm(h)."""
    rows = h.numel() // h.shape[-1] if h.shape[-1] else 0
    _buf("h", h, 0)
    _buf("delta", delta, rows * h.shape[-1], cols=h.shape[-1])
    _buf("w", w, h.shape[-1])
    _buf("out", out, rows * h.shape[-1], cols=h.shape[-1])
    _cuda(h, delta, w, out)
    _run("ckv_add_rmsnorm", _ptr(h), _ptr(delta), _ptr(w), _ptr(out), rows, h.shape[-1], float(eps),
         _stream())
    return out


def linear_partial(x: torch.Tensor, w: torch.Tensor, exch, buf: int) -> None:
    """Row-parallel GEMM into this rank's partial buffer `buf`, then a signal to every rank."""
    _cuda(x, w)
    _bf16(x, w)
    _contig(x, w)
    m, k = x.shape
    n = w.shape[0]
    tp = exch.tp
    _run("ckv_linear_partial", _ptr(x), _ptr(w), _ptr(exch.part[buf]), m, n, k, _ptr(exch.flag_tab),
         _ptr(exch.push_ticket), tp.rank, tp.size, _stream(), flops=2.0 * m * n * k)


def reduce_add_gather(exch, buf: int, pair: int, m: int) -> None:
    """The ranks' partial rows in buffer `buf` (read over NVLink by the owning ranks) added to
    h[pair] and gathered into every rank's h[pair] (one exchange: epoch + 1)."""
    exch.epoch += 1
    tp = exch.tp
    _run("ckv_reduce_add_gather", _ptr(exch.part_tab[buf]), tp.rank, tp.size, m, exch.hidden,
         _ptr(exch.h[pair]), _ptr(exch.h_tab[pair]), _ptr(exch.recv_cnt), _ptr(exch.gather_cnt),
         _ptr(exch.gather_tab), _ptr(exch.reduce_ticket), exch.epoch & 0xFFFFFFFF, _stream(),
         nbytes=2.0 * (tp.size - 1) / tp.size * m * exch.hidden * 2)


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    k = x.shape[-1]
    m = x.numel() // k if k else 0
    _buf("x", x, 0)
    n = _weight("w", w, None, k)
    if bias is not None:
        _buf("bias", bias, n)
    if out is not None:
        _buf("out", out, m * n, cols=n)
    _cuda(x, w, bias, out)
    out = torch.empty((*x.shape[:-1], n), dtype=BF16, device=x.device) if out is None else out
    _run("ckv_linear", _ptr(x), _ptr(w), _ptr(bias), _ptr(out), m, n, k, _stream(), flops=2.0 * m * n * k)
    return out


def linear_residual(x: torch.Tensor, w: torch.Tensor, h: torch.Tensor, m: int | None = None) -> torch.Tensor:
    """h[:m] = bf16(h + bf16(x[:m] W^T)) (m defaults to all rows of x)."""
    k = x.shape[-1]
    m = (x.numel() // k if k else 0) if m is None else m
    _buf("x", x, m * k)
    n = _weight("w", w, None, k)
    _buf("h", h, m * n, cols=n)
    _cuda(x, w, h)
    _run("ckv_linear_residual", _ptr(x), _ptr(w), _ptr(h), m, n, k, _stream(), flops=2.0 * m * n * k)
    return h


def linear_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, out: torch.Tensor, m: int | None = None) -> torch.Tensor:
    """out[:m] = SwiGLU of x[:m] through the interleaved gate/up weight [2*inter][k]."""
    k = x.shape[-1]
    m = (x.numel() // k if k else 0) if m is None else m
    _buf("x", x, m * k)
    n2 = _weight("w_gate_up", w_gate_up, None, k)
    _buf("out", out, m * (n2 // 2), cols=n2 // 2)
    _cuda(x, w_gate_up, out)
    _run("ckv_linear_swiglu", _ptr(x), _ptr(w_gate_up), _ptr(out), m, n2 // 2, k, _stream(),
         flops=2.0 * m * n2 * k)
    return out


def qkv_rope(x, w_qkv, b_qkv, m, col_begin, col_end, n_q_heads, n_kv_heads, head_dim, positions,
             rope_tab, q_out=None, k_cache=None, v_cache=None, k_compact=None, v_compact=None) -> None:
    """Columns [col_begin, col_end) of the QKV projection of x[:m] with bias and RoPE at
    positions[:m]: q -> q_out, k/v -> the caches [H, n_ctx, D] and/or compact [m, H*D] rows."""
    k = x.shape[-1]
    _buf("x", x, m * k)
    n = _weight("w_qkv", w_qkv, (n_q_heads + 2 * n_kv_heads) * head_dim, k)
    if not 0 <= col_begin <= col_end <= n:
        raise ValueError(f"columns [{col_begin}, {col_end}) outside the {n} rows of w_qkv")
    if b_qkv is not None:
        _buf("b_qkv", b_qkv, n)
    _buf("positions", positions, m, dtype=torch.int32)
    _rope_tab(rope_tab, head_dim)
    if q_out is not None:
        _buf("q_out", q_out, m * n_q_heads * head_dim)
    n_ctx = k_cache.shape[1] if k_cache is not None else 0
    for name, c in (("k_cache", k_cache), ("v_cache", v_cache)):
        if c is not None:
            _cache(name, c, n_kv_heads, head_dim)
            if c.shape[1] != n_ctx:
                raise ValueError("k_cache and v_cache differ in length")
    for name, c in (("k_compact", k_compact), ("v_compact", v_compact)):
        if c is not None:
            _buf(name, c, m * n_kv_heads * head_dim)
    _cuda(x, w_qkv, b_qkv, positions, rope_tab, q_out, k_cache, v_cache, k_compact, v_compact)
    _run("ckv_qkv_rope", _ptr(x), _ptr(w_qkv), _ptr(b_qkv), m, x.shape[-1], col_begin, col_end,
              n_q_heads, n_kv_heads, head_dim, _ptr(positions), _ptr(rope_tab), rope_tab.shape[0],
              _ptr(q_out), _ptr(k_cache), _ptr(v_cache), n_ctx, _ptr(k_compact), _ptr(v_compact),
              _stream(), flops=2.0 * m * (col_end - col_begin) * x.shape[-1])


def attention_workspace_bytes(m: int, n_q_heads: int, n_kv_heads: int, head_dim: int, n_ctx: int) -> int:
    """Bytes of attention workspace for a shape: 256 bytes of scheduler words, plus the
    key-split partials when the shape benefits from splitting the keys."""
    return int(_lib.load().ckv_attention_workspace_size(m, n_q_heads, n_kv_heads, head_dim, n_ctx))


ATTN_SCHED_BYTES = 256
_attn_scratch: dict[torch.device, torch.Tensor] = {}


def attention_workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A zeroed attention workspace of at least `nbytes`, kept per device and grown on
    demand.  Every launch leaves its scheduler words at zero again, so the buffer is
    reused as it is by later launches in stream order."""
    ws = _attn_scratch.get(device)
    if ws is None or ws.numel() < nbytes:
        ws = _attn_scratch[device] = torch.zeros(max(nbytes, ATTN_SCHED_BYTES), dtype=torch.uint8, device=device)
    return ws


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, positions: torch.Tensor,
              out: torch.Tensor, m: int | None = None, scale: float | None = None,
              flops: float = 0.0, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """q/out [m, Hq, D]; caches [H, n_ctx, D]; key j visible to row i iff j <= positions[i].
    `workspace` must have been zeroed once when allocated (``attention_workspace``);
    without it the per-device scratch buffer is used."""
    if k_cache.dim() != 3:
        raise ValueError(f"k_cache: expected shape (H, n_ctx, D), got {tuple(k_cache.shape)}")
    H, n_ctx, D = k_cache.shape
    m = q.shape[0] if m is None else m
    Hq = q.shape[-2] if q.dim() == 3 else q.shape[-1] // D
    _cache("k_cache", k_cache, H, D)
    _cache("v_cache", v_cache, H, D)
    if v_cache.shape[1] != n_ctx:
        raise ValueError("k_cache and v_cache differ in length")
    _buf("q", q, m * Hq * D)
    _buf("out", out, m * Hq * D)
    _buf("positions", positions, m, dtype=torch.int32)
    _cuda(q, k_cache, v_cache, positions, out, workspace)
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    need = attention_workspace_bytes(m, Hq, H, D, n_ctx)
    if workspace is None:
        workspace = attention_workspace(need, q.device)
    ws_bytes = workspace.numel() * workspace.element_size()
    if ws_bytes == 0:  # an empty workspace: static scheduling, no key split
        workspace = None
    kernels = int(_lib.load().ckv_attention_launches(m, Hq, H, D, n_ctx, ws_bytes))
    _run("ckv_attention", _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(positions), _ptr(out), m, Hq,
         H, D, n_ctx, float(scale), _ptr(workspace), ws_bytes, _stream(), flops=flops,
         kernels=max(kernels, 1))
    return out


def gemv(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out [m, n] = bf16(x W^T) for m = x rows <= 8 (lm_head on the logit rows)."""
    m, k = _rows_k(x)
    n = _weight("w", w, None, k)
    if out is not None:
        _buf("out", out, m * n, cols=n)
    _cuda(x, w, out)
    out = torch.empty((m, w.shape[0]), dtype=BF16, device=x.device) if out is None else out
    _run("ckv_gemv", _ptr(x), _ptr(w), _ptr(out), m, w.shape[0], k, _stream(),
         flops=2.0 * m * w.shape[0] * k, nbytes=2.0 * w.shape[0] * k)
    return out


def gemv_residual(x: torch.Tensor, w: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
    """h[:m] = bf16(h + bf16(x W^T)) for m = x rows <= 8 (decode)."""
    m, k = _rows_k(x)
    n = _weight("w", w, None, k)
    _buf("h", h, m * n, cols=n)
    _cuda(x, w, h)
    _run("ckv_gemv_residual", _ptr(x), _ptr(w), _ptr(h), m, n, k, _stream(),
         flops=2.0 * m * n * k, nbytes=2.0 * n * k)
    return h


GEMV_NORM_MAX_ROWS, GEMV_NORM_MAX_K = 4, 5120  # the fused-RMSNorm GEMVs' limits


def gemv_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, out: torch.Tensor,
                norm_w: torch.Tensor | None = None, eps: float = 1e-6) -> torch.Tensor:
    """SwiGLU of the interleaved gate/up projection for m = x rows <= 8 (decode).  With
    `norm_w`, x is the hidden state h and the projection takes RMSNorm(h) (m <= 4)."""
    m, k = _rows_k(x)
    inter = _weight("w_gate_up", w_gate_up, None, k) // 2
    _buf("out", out, m * inter, cols=inter)
    if norm_w is not None:
        _buf("norm_w", norm_w, k)
    _cuda(x, w_gate_up, out, norm_w)
    if norm_w is None:
        _run("ckv_gemv_swiglu", _ptr(x), _ptr(w_gate_up), _ptr(out), m, inter, k, _stream(),
             flops=2.0 * m * 2 * inter * k, nbytes=2.0 * 2 * inter * k)
    else:
        _run("ckv_gemv_swiglu_rmsnorm", _ptr(x), _ptr(norm_w), float(eps), _ptr(w_gate_up), _ptr(out), m, inter,
             k, _stream(), flops=2.0 * m * 2 * inter * k, nbytes=2.0 * 2 * inter * k)
    return out


def gemv_qkv_rope(x: torch.Tensor, w_qkv: torch.Tensor, b_qkv: torch.Tensor, Hq: int, Hk: int, D: int,
                  positions: torch.Tensor, rope_tab: torch.Tensor, q_out: torch.Tensor,
                  k_cache: torch.Tensor, v_cache: torch.Tensor, norm_w: torch.Tensor | None = None,
                  eps: float = 1e-6) -> None:
    """q/k/v of m = x rows <= 8 with bias and RoPE; k, v written into the caches (decode).
    With `norm_w`, x is the hidden state h and the projection takes RMSNorm(h) (m <= 4)."""
    m, k = _rows_k(x)
    _weight("w_qkv", w_qkv, (Hq + 2 * Hk) * D, k)
    _buf("b_qkv", b_qkv, (Hq + 2 * Hk) * D)
    _buf("positions", positions, m, dtype=torch.int32)
    _rope_tab(rope_tab, D)
    _buf("q_out", q_out, m * Hq * D)
    _cache("k_cache", k_cache, Hk, D)
    _cache("v_cache", v_cache, Hk, D)
    if v_cache.shape[1] != k_cache.shape[1]:
        raise ValueError("k_cache and v_cache differ in length")
    if norm_w is not None:
        _buf("norm_w", norm_w, k)
    _cuda(x, w_qkv, b_qkv, positions, rope_tab, q_out, k_cache, v_cache, norm_w)
    n_ctx = k_cache.shape[1]
    args = (_ptr(w_qkv), _ptr(b_qkv), m, k, Hq, Hk, D, _ptr(positions), _ptr(rope_tab), rope_tab.shape[0],
            _ptr(q_out), _ptr(k_cache), _ptr(v_cache), n_ctx, _stream())
    work = dict(flops=2.0 * m * w_qkv.shape[0] * k, nbytes=2.0 * w_qkv.shape[0] * k)
    if norm_w is None:
        _run("ckv_gemv_qkv_rope", _ptr(x), *args, **work)
    else:
        _run("ckv_gemv_qkv_rope_rmsnorm", _ptr(x), _ptr(norm_w), float(eps), *args, **work)


def greedy_next(row: torch.Tensor, token: torch.Tensor, position: torch.Tensor | None = None) -> torch.Tensor:
    """token[0] = argmax of the bf16 logits `row` (torch.argmax's order: NaN first, ties to
    the lower index); with `position`, position[0] += 1 in the same launch (the greedy
    decode step of torch_engine.py:196-197).  Both are int32 device tensors."""
    _buf("row", row, 1)
    _buf("token", token, 1, dtype=torch.int32)
    if position is not None:
        _buf("position", position, 1, dtype=torch.int32)
    _cuda(row, token, position)
    _run("ckv_greedy_next", _ptr(row), row.numel(), _ptr(token), _ptr(position), _stream())
    return token


def log_softmax(row: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _buf("row", row, 0)
    if out is not None:
        _buf("out", out, row.numel(), dtype=torch.float32)
    _cuda(row, out)
    out = torch.empty(row.numel(), dtype=torch.float32, device=row.device) if out is None else out
    _run("ckv_log_softmax", _ptr(row), row.numel(), _ptr(out), _stream())
    return out
