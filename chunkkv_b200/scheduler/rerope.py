"""Rotary position helpers for moving cached keys (drop-in for chunkkv.scheduler.rerope).

Same API as src/chunkkv/scheduler/rerope.py:16-61 (RopeSpec, apply_rope,
shift_keys), on torch CUDA tensors and this package's kernels instead of MLX.
RoPE rotates each frequency pair (j, j + dims/2) by position * inv_freq[j];
rotations compose, so a key computed at p moves to p + delta by rotating it by
delta.  Half-split layout only, no scaling; dims < head_dim rotates the first
`dims` dimensions and copies the rest.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from chunkkv_b200 import ops


@dataclass(frozen=True)
class RopeSpec:
    dims: int
    base: float
    traditional: bool = False

    @classmethod
    def from_model(cls, model) -> "RopeSpec":
        """From an HF config-carrying model (or a config): rejects rope scaling like the reference."""
        cfg = getattr(model, "config", model)
        scaling = getattr(cfg, "rope_scaling", None) or {}
        if scaling and scaling.get("rope_type", scaling.get("type", "default")) != "default":
            raise NotImplementedError("rope_scaling is not supported in v0")
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        base = getattr(cfg, "rope_theta", None) or scaling.get("rope_theta") or cfg.rope_parameters["rope_theta"]
        return cls(dims=head_dim, base=float(base), traditional=bool(getattr(cfg, "rope_traditional", False)))


_INV: dict = {}


def _inv_freq(spec: RopeSpec, device) -> torch.Tensor:
    key = (spec.dims, spec.base, str(device))
    t = _INV.get(key)
    if t is None:
        half = spec.dims // 2
        t = torch.pow(spec.base, -torch.arange(0, half, dtype=torch.float32, device=device) * 2.0 / spec.dims)
        _INV[key] = t
    return t


def _check(spec: RopeSpec, x: torch.Tensor) -> None:
    if spec.traditional:
        raise NotImplementedError("traditional RoPE layout is not supported in v0")
    if spec.dims > x.shape[-1]:
        raise ValueError(f"rotary dims {spec.dims} exceed head_dim {x.shape[-1]}")


def apply_rope(x: torch.Tensor, positions: torch.Tensor, spec: RopeSpec) -> torch.Tensor:
    """RoPE of x (B, H, L, D) at arbitrary (possibly non-contiguous) positions (L,),
    rotated in fp32 and returned in x's dtype (bf16 or fp32; others raise
    NotImplementedError), as rerope.py:36-53 does."""
    _check(spec, x)
    pos = torch.as_tensor(positions, device=x.device)
    return ops.apply_rope(x.contiguous(), pos, _inv_freq(spec, x.device), rot_dims=spec.dims)


def shift_keys(keys: torch.Tensor, delta: int, spec: RopeSpec) -> torch.Tensor:
    """Move already-rotated keys (B, H, L, D) by `delta` positions, rotated in fp32 and
    returned in the keys' dtype (bf16 or fp32; others raise NotImplementedError);
    delta 0 returns `keys` itself (rerope.py:56-61)."""
    if delta == 0:
        return keys
    _check(spec, keys)
    return ops.shift_keys(keys.contiguous(), int(delta), _inv_freq(spec, keys.device), rot_dims=spec.dims)
