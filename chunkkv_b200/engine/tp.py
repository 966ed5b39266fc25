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

    def __init__(self, group=None, fused: bool = True):
        """`fused`: o_proj / down_proj exchange their partial rows over NVLink peer memory
        (`ckv_linear_partial` + `ckv_reduce_add_gather`); False: NCCL all-reduce.  The
        peer-memory exchange measured faster with 2, 4 and 8 ranks (32B prefill: 227 vs
        235 ms, 125 vs 129 ms, 82 vs 88 ms)."""
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("TensorParallel needs an initialised torch.distributed process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.fused = bool(fused)
        self.bytes_reduced = 0  # running total of all-reduced bytes (bus-bandwidth accounting)
        self._exchange: "PeerExchange | None" = None

    def exchange(self, rows: int, hidden: int, device) -> "PeerExchange":
        """The peer-memory buffers for at least `rows` rows (collective when it grows)."""
        ex = self._exchange
        if ex is None or ex.rows < rows or ex.hidden != hidden:
            if ex is not None:
                ex.close()
            cap = max(rows, 256)
            cap = (cap + 127) // 128 * 128
            self._exchange = ex = PeerExchange(self, cap, hidden, device)
        return ex

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


class _DeviceArray:
    """Raw device memory as a torch tensor (no copy) via __cuda_array_interface__."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3}


class PeerExchange:
    """Buffers of the NVLink exchange (`ckv_linear_partial` + `ckv_reduce_add_gather`),
    allocated by every rank and mapped into every other rank with CUDA IPC:

      part[2]  this rank's partial rows, [rows][hidden] bf16, alternating between exchanges
      h[2], x[2]  the residual stream (gathered from the owning ranks) and the normed rows
               (computed locally), [rows][hidden] bf16; the pair in use flips when the
               layer-1 selection shrinks the rows into the other pair
      ctl      uint32 partial counters [ranks], gather counters [ranks], two CTA tickets

    Every rank must make the same exchanges in the same order (they do: each rank runs
    the same prefill).  `epoch` counts the exchanges made so far."""

    MAX_RANKS = 8
    CTL_BYTES = 256

    def __init__(self, tp: TensorParallel, rows: int, hidden: int, device):
        from chunkkv_b200 import _lib

        if tp.size > self.MAX_RANKS:
            raise NotImplementedError(f"at most {self.MAX_RANKS} ranks")
        self.tp, self.rows, self.hidden, self.device = tp, rows, hidden, torch.device(device)
        self.epoch = 0
        self.recv_toggle = 0
        T, row_bytes = tp.size, rows * hidden * 2
        sizes = {"part0": row_bytes, "part1": row_bytes, "hx": 4 * row_bytes, "ctl": self.CTL_BYTES}
        self._local: dict[str, int] = {}
        handles: dict[str, bytes] = {}
        lib = _lib.load()
        import ctypes

        for name, nb in sizes.items():
            ptr = ctypes.c_void_p()
            h = ctypes.create_string_buffer(64)
            _lib.call("ckv_ipc_alloc", nb, ctypes.byref(ptr), h)
            self._local[name] = ptr.value
            handles[name] = h.raw
        everyone: list[dict[str, bytes]] = [None] * T  # type: ignore[list-item]
        dist.all_gather_object(everyone, handles, group=tp.group)
        self._opened: list[int] = []
        base: dict[str, list[int]] = {name: [0] * T for name in sizes}
        for q in range(T):
            for name in sizes:
                if q == tp.rank:
                    base[name][q] = self._local[name]
                    continue
                ptr = ctypes.c_void_p()
                _lib.call("ckv_ipc_open", everyone[q][name], ctypes.byref(ptr))
                base[name][q] = ptr.value
                self._opened.append(ptr.value)
        del lib

        def table(vals):
            return torch.tensor(vals, dtype=torch.int64).view(torch.uint64).to(self.device)

        self.part_tab = [table(base["part0"]), table(base["part1"])]
        self.flag_tab = table(base["ctl"])                        # partial counters at offset 0
        self.gather_tab = table([b + 4 * self.MAX_RANKS for b in base["ctl"]])
        self.h_tab = [table([b + k * row_bytes for b in base["hx"]]) for k in (0, 2)]
        bf = torch.bfloat16

        def view(ptr, nbytes, shape, dtype):
            return torch.as_tensor(_DeviceArray(ptr, nbytes), device=self.device).view(dtype).view(shape)

        hx = self._local["hx"]
        self.h = [view(hx + k * row_bytes, row_bytes, (rows, hidden), bf) for k in (0, 2)]
        self.x = [view(hx + k * row_bytes, row_bytes, (rows, hidden), bf) for k in (1, 3)]
        self.part = [view(self._local[f"part{i}"], row_bytes, (rows, hidden), bf) for i in (0, 1)]
        ctl = view(self._local["ctl"], self.CTL_BYTES, (self.CTL_BYTES // 4,), torch.int32)
        self.recv_cnt = ctl[:self.MAX_RANKS]
        self.gather_cnt = ctl[self.MAX_RANKS:2 * self.MAX_RANKS]
        self.push_ticket = ctl[2 * self.MAX_RANKS:2 * self.MAX_RANKS + 1]
        self.reduce_ticket = ctl[2 * self.MAX_RANKS + 1:2 * self.MAX_RANKS + 2]
        dist.barrier(group=tp.group)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: all ranks call it)."""
        from chunkkv_b200 import _lib

        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.tp.group)
        for p in self._opened:
            _lib.call("ckv_ipc_close", p)
        dist.barrier(group=self.tp.group)
        for p in self._local.values():
            _lib.call("ckv_ipc_free", p)
        self._opened, self._local = [], {}
