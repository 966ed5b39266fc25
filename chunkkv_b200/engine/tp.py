"""Tensor-parallel group of the blend prefill (one process per GPU, NCCL over NVLink).

The reference runs one model on one device (torch_engine.py:18-207); a model whose
weights and 32k-token K/V do not fit one request per GPU is split by KV head:
rank r computes KV heads [r*H/T, (r+1)*H/T) with their query heads, and its share
of the MLP's intermediate rows.  Everything position-wise (embedding, RMSNorm,
residual stream, logits, the selection) is replicated; the exchange steps are

  * after o_proj and after down_proj (row-parallel): a sum of the ranks' bf16
    partial outputs [M, hidden] (all-reduce), then the residual add + RMSNorm;
  * at layer 1: a sum of the ranks' fp32 deviation scores [2, n_ctx] (each rank
    scores its own heads), then the same deterministic selection on every rank.

NCCL returns the identical reduced buffer on every rank, so the replicated
state (h, the selection) stays bit-identical across ranks.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class TensorParallel:
    """A process group used as the engine's tensor-parallel group."""

    def __init__(self, group=None):
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("TensorParallel needs an initialised torch.distributed process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.bytes_reduced = 0  # running total of all-reduced bytes (bus-bandwidth accounting)

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over the group, ordered on the current stream.  Under an
        `ops.LaunchTimer` the call is timed like a kernel, as "nccl_all_reduce" with
        its bus bytes 2 (T-1)/T x size."""
        if self.size == 1:
            return t
        from chunkkv_b200 import ops

        timer = ops._TIMER
        nbytes = t.numel() * t.element_size()
        if timer is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        if timer is not None:
            e1.record()
            timer.records.append(("nccl_all_reduce", 0.0, 2.0 * (self.size - 1) / self.size * nbytes, e0, e1))
            timer.kernels["nccl_all_reduce"] = 0  # NCCL's kernels, not this library's
        self.bytes_reduced += nbytes
        return t

    def __repr__(self) -> str:
        return f"TensorParallel(rank={self.rank}, size={self.size})"
