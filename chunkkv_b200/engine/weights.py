"""Qwen2-family shapes, seeded random weights and the packed layout of the CUDA engine.

`random_state_dict` produces Hugging Face `Qwen2ForCausalLM` parameter names, so
the same tensors can be loaded into the reference's HF model (for parity) and
packed for this engine.  Packing (one-time, at load):
  w_qkv  [Hq*D + 2*H*D, hidden]  rows q | k | v, with the matching bias
  w_o    [hidden, Hq*D]
  w_gu   [2*inter, hidden]        gate/up interleaved in 128-row blocks
                                  (block b = gate rows 128b.. then up rows 128b..)
  w_down [hidden, inter]

Tensor parallel (`tp_size` > 1, rank `tp_rank`): rank r keeps KV heads
[r*H/T, (r+1)*H/T) with their query heads, the same slice of q/k/v rows and
of the o_proj columns, and intermediate rows [r*I/T, (r+1)*I/T) of gate/up with
the matching down_proj columns (column-parallel QKV and gate/up, row-parallel
o_proj and down_proj).  Embedding, norms and lm_head are replicated.  The
packed `shape` of a rank is its local shape (`tp_local`).
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch

GU_BLOCK = 128  # rows per gate (and per up) block in the interleaved gate/up weight


@dataclass(frozen=True)
class Qwen2Shape:
    name: str
    n_layers: int
    hidden: int
    n_heads: int
    n_kv: int
    head_dim: int
    inter: int
    vocab: int
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    tied: bool = False

    def truncated(self, n_layers: int) -> "Qwen2Shape":
        return replace(self, name=f"{self.name}-L{n_layers}", n_layers=n_layers)

    def tp_local(self, tp_size: int) -> "Qwen2Shape":
        """The shape one of `tp_size` tensor-parallel ranks computes: its share of the
        query/KV heads and of the intermediate size; hidden, vocab, layers unchanged."""
        if tp_size == 1:
            return self
        if self.n_kv % tp_size or self.inter % tp_size or (self.inter // tp_size) % GU_BLOCK:
            raise NotImplementedError(
                f"{self.name}: {self.n_kv} KV heads / intermediate {self.inter} do not split {tp_size} ways "
                f"(need whole KV heads and {GU_BLOCK}-row gate/up blocks per rank)")
        return replace(self, name=f"{self.name}-tp{tp_size}", n_heads=self.n_heads // tp_size,
                       n_kv=self.n_kv // tp_size, inter=self.inter // tp_size)

    def hf_config(self):
        from transformers import Qwen2Config

        return Qwen2Config(
            vocab_size=self.vocab, hidden_size=self.hidden, intermediate_size=self.inter,
            num_hidden_layers=self.n_layers, num_attention_heads=self.n_heads,
            num_key_value_heads=self.n_kv, head_dim=self.head_dim, max_position_embeddings=131072,
            rope_theta=self.rope_theta, rms_norm_eps=self.rms_eps, tie_word_embeddings=self.tied,
            hidden_act="silu", attention_dropout=0.0, use_sliding_window=False)

    @property
    def kv_bytes_per_token(self) -> int:
        """bf16 K+V bytes of one token over all layers."""
        return self.n_layers * 2 * self.n_kv * self.head_dim * 2

    def linear_flops_per_token_layer(self) -> int:
        qkv = (self.n_heads + 2 * self.n_kv) * self.head_dim
        return 2 * self.hidden * (qkv + self.n_heads * self.head_dim + 3 * self.inter)


SHAPES = {
    # small shape for the fast tests (GQA 2:1, head_dim 64)
    "tiny": Qwen2Shape("tiny", n_layers=4, hidden=256, n_heads=4, n_kv=2, head_dim=64, inter=512,
                       vocab=1024),
    # GQA 7:1 at head_dim 128, like the 7B, but small
    "tiny7": Qwen2Shape("tiny7", n_layers=3, hidden=896, n_heads=7, n_kv=1, head_dim=128, inter=1024,
                        vocab=2048),
    "qwen2.5-0.5b": Qwen2Shape("qwen2.5-0.5b", n_layers=24, hidden=896, n_heads=14, n_kv=2,
                               head_dim=64, inter=4864, vocab=151936, tied=True),
    "qwen2.5-7b": Qwen2Shape("qwen2.5-7b", n_layers=28, hidden=3584, n_heads=28, n_kv=4, head_dim=128,
                             inter=18944, vocab=152064),
    "qwen2.5-32b": Qwen2Shape("qwen2.5-32b", n_layers=64, hidden=5120, n_heads=40, n_kv=8,
                              head_dim=128, inter=27648, vocab=152064),
}


def param_shapes(shape: Qwen2Shape) -> list[tuple[str, tuple[int, ...]]]:
    """HF parameter names and shapes, in a fixed order (the order random values are drawn in)."""
    D, H, Hq = shape.head_dim, shape.n_kv, shape.n_heads
    out = [("model.embed_tokens.weight", (shape.vocab, shape.hidden))]
    for i in range(shape.n_layers):
        p = f"model.layers.{i}."
        out += [
            (p + "input_layernorm.weight", (shape.hidden,)),
            (p + "self_attn.q_proj.weight", (Hq * D, shape.hidden)),
            (p + "self_attn.q_proj.bias", (Hq * D,)),
            (p + "self_attn.k_proj.weight", (H * D, shape.hidden)),
            (p + "self_attn.k_proj.bias", (H * D,)),
            (p + "self_attn.v_proj.weight", (H * D, shape.hidden)),
            (p + "self_attn.v_proj.bias", (H * D,)),
            (p + "self_attn.o_proj.weight", (shape.hidden, Hq * D)),
            (p + "post_attention_layernorm.weight", (shape.hidden,)),
            (p + "mlp.gate_proj.weight", (shape.inter, shape.hidden)),
            (p + "mlp.up_proj.weight", (shape.inter, shape.hidden)),
            (p + "mlp.down_proj.weight", (shape.hidden, shape.inter)),
        ]
    out.append(("model.norm.weight", (shape.hidden,)))
    if not shape.tied:
        out.append(("lm_head.weight", (shape.vocab, shape.hidden)))
    return out


def random_state_dict(shape: Qwen2Shape, seed: int = 0, dtype=torch.bfloat16, device="cpu",
                      std: float = 0.02, bias_std: float = 0.02, emb_std: float = 1.0,
                      norm_jitter: float = 0.1) -> dict[str, torch.Tensor]:
    """Seeded random weights with HF names, drawn in fp32 from one generator in
    `param_shapes` order and cast to `dtype`.  To give two engines identical
    values, make the bf16 dict once and upcast it where fp32 is wanted.
    Embeddings ~ N(0, emb_std), linears ~ N(0, std), biases ~ N(0, bias_std),
    norm weights ~ 1 + U(-jitter, jitter)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    sd: dict[str, torch.Tensor] = {}
    for name, shp in param_shapes(shape):
        if name.endswith("layernorm.weight") or name == "model.norm.weight":
            t = 1.0 + (torch.rand(shp, generator=gen, device=device) * 2 - 1) * norm_jitter
        elif name.endswith(".bias"):
            t = torch.randn(shp, generator=gen, device=device) * bias_std
        elif "embed_tokens" in name or name == "lm_head.weight":
            t = torch.randn(shp, generator=gen, device=device) * (emb_std if "embed" in name else std)
        else:
            t = torch.randn(shp, generator=gen, device=device) * std
        sd[name] = t.to(dtype)
    if shape.tied:
        sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    return sd


def hf_model(shape: Qwen2Shape, state_dict: dict[str, torch.Tensor], dtype=torch.float32):
    """A Hugging Face Qwen2ForCausalLM holding `state_dict` (for the reference engine)."""
    from transformers import Qwen2ForCausalLM

    model = Qwen2ForCausalLM(shape.hf_config()).to(dtype)
    sd = {k: v.to(dtype) for k, v in state_dict.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    bad = [m for m in missing if not (shape.tied and m == "lm_head.weight")]
    if bad or unexpected:
        raise ValueError(f"state dict mismatch: missing {bad}, unexpected {unexpected}")
    if shape.tied:
        model.tie_weights()
    return model.eval()


@dataclass
class LayerWeights:
    ln1: torch.Tensor
    w_qkv: torch.Tensor
    b_qkv: torch.Tensor
    w_o: torch.Tensor
    ln2: torch.Tensor
    w_gu: torch.Tensor
    w_down: torch.Tensor


@dataclass
class PackedQwen2:
    shape: Qwen2Shape  # the local shape of this rank when tensor parallel
    embed: torch.Tensor
    layers: list[LayerWeights]
    norm: torch.Tensor
    lm_head: torch.Tensor
    tp_rank: int = 0
    tp_size: int = 1

    @property
    def device(self) -> torch.device:
        return self.embed.device

    def nbytes(self) -> int:
        ts = [self.embed, self.norm] + ([] if self.lm_head is self.embed else [self.lm_head])
        for lw in self.layers:
            ts += [lw.ln1, lw.w_qkv, lw.b_qkv, lw.w_o, lw.ln2, lw.w_gu, lw.w_down]
        return sum(t.numel() * t.element_size() for t in ts)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    inter, hidden = gate.shape
    if inter % GU_BLOCK:
        raise NotImplementedError(f"intermediate size {inter} is not a multiple of {GU_BLOCK}")
    g = gate.reshape(inter // GU_BLOCK, GU_BLOCK, hidden)
    u = up.reshape(inter // GU_BLOCK, GU_BLOCK, hidden)
    return torch.stack([g, u], dim=1).reshape(2 * inter, hidden).contiguous()


def pack(shape: Qwen2Shape, sd: dict[str, torch.Tensor], device="cuda", tp_rank: int = 0,
         tp_size: int = 1) -> PackedQwen2:
    """Pack HF-named weights into the engine layout as contiguous bf16 on `device`;
    with tp_size > 1, only rank `tp_rank`'s shard (module docstring)."""
    loc = shape.tp_local(tp_size)
    D, r = shape.head_dim, tp_rank
    qs = slice(r * loc.n_heads * D, (r + 1) * loc.n_heads * D)
    ks = slice(r * loc.n_kv * D, (r + 1) * loc.n_kv * D)
    fs = slice(r * loc.inter, (r + 1) * loc.inter)

    def get(name, rows=slice(None), cols=slice(None)):
        t = sd[name]
        t = t[rows] if t.dim() == 1 else t[rows, cols]
        return t.to(device=device, dtype=torch.bfloat16).contiguous()

    layers = []
    for i in range(shape.n_layers):
        p = f"model.layers.{i}."
        w_qkv = torch.cat([get(p + "self_attn.q_proj.weight", qs), get(p + "self_attn.k_proj.weight", ks),
                           get(p + "self_attn.v_proj.weight", ks)], 0).contiguous()
        b_qkv = torch.cat([get(p + "self_attn.q_proj.bias", qs), get(p + "self_attn.k_proj.bias", ks),
                           get(p + "self_attn.v_proj.bias", ks)], 0).contiguous()
        layers.append(LayerWeights(
            ln1=get(p + "input_layernorm.weight"), w_qkv=w_qkv, b_qkv=b_qkv,
            w_o=get(p + "self_attn.o_proj.weight", slice(None), qs),
            ln2=get(p + "post_attention_layernorm.weight"),
            w_gu=interleave_gate_up(get(p + "mlp.gate_proj.weight", fs), get(p + "mlp.up_proj.weight", fs)),
            w_down=get(p + "mlp.down_proj.weight", slice(None), fs)))
    embed = get("model.embed_tokens.weight")
    lm = embed if shape.tied else get("lm_head.weight")
    return PackedQwen2(loc, embed, layers, get("model.norm.weight"), lm, tp_rank, tp_size)


def random_packed(shape: Qwen2Shape, seed: int = 0, device="cuda", std: float = 0.02,
                  tp_rank: int = 0, tp_size: int = 1) -> PackedQwen2:
    """Random weights generated directly on the device, already packed (for large shapes:
    no host copy).  Same distributions as random_state_dict but a different stream of
    values (device generator), so not comparable with a CPU-generated state dict.
    With tp_size > 1 each rank draws only its shard, from a generator seeded by
    (seed, rank); the replicated embedding, norms and lm_head come from `seed`
    alone, so they are identical on every rank."""
    gen = torch.Generator(device=device).manual_seed(seed)
    rep = gen
    if tp_size > 1:
        rep = torch.Generator(device=device).manual_seed(seed)
        gen = torch.Generator(device=device).manual_seed(seed * 1009 + 1 + tp_rank)
    loc = shape.tp_local(tp_size)
    bf = torch.bfloat16

    def randn(*shp, s=std, g=None):
        return (torch.randn(shp, generator=g or gen, device=device, dtype=torch.float32) * s).to(bf)

    def norm_w(n):
        return (1.0 + (torch.rand(n, generator=rep, device=device) * 2 - 1) * 0.1).to(bf)

    D, H, Hq, hid = loc.head_dim, loc.n_kv, loc.n_heads, loc.hidden
    qkv = (Hq + 2 * H) * D
    layers = []
    for _ in range(shape.n_layers):
        layers.append(LayerWeights(
            ln1=norm_w(hid), w_qkv=randn(qkv, hid), b_qkv=randn(qkv), w_o=randn(hid, Hq * D),
            ln2=norm_w(hid), w_gu=randn(2 * loc.inter, hid), w_down=randn(hid, loc.inter)))
    embed = randn(shape.vocab, hid, s=1.0, g=rep)
    lm = embed if shape.tied else randn(shape.vocab, hid, g=rep)
    return PackedQwen2(loc, embed, layers, norm_w(hid), lm, tp_rank, tp_size)
