"""Pinned host staging for the engine's and the store's small uploads and readbacks.

Several small host arrays (token ids, flags, chunk tables, page pointers) go to
the device in ONE copy from a reused pinned buffer; an event recorded after the
copy guards the buffer's reuse, so no call waits for the GPU unless the previous
copy out of the same buffer is still in flight.
"""

from __future__ import annotations

import numpy as np
import torch

_ALIGN = 16


class Staging:
    """`slots` pinned host buffers used round robin, each guarded by the event recorded
    after its last copy: a call waits only when the copy made `slots` calls ago out of
    the same buffer has not run yet (with one slot: the previous copy)."""

    def __init__(self, slots: int = 1):
        self.hosts: list[torch.Tensor | None] = [None] * slots
        self.events: list[torch.cuda.Event | None] = [None] * slots
        # per slot: the device buffer of the last upload and its views, reused by the next
        # upload of the same layout (a copy into it is ordered after the kernels that read
        # it on the same stream)
        self.dev: list[tuple | None] = [None] * slots
        self.i = 0

    def get(self, nbytes: int) -> torch.Tensor:
        self.i = (self.i + 1) % len(self.hosts)
        ev, host = self.events[self.i], self.hosts[self.i]
        if ev is not None:
            ev.synchronize()
        if host is None or host.numel() < nbytes:
            host = self.hosts[self.i] = torch.empty(max(nbytes, 1 << 12) * 2, dtype=torch.uint8,
                                                    pin_memory=True)
        return host[:nbytes]

    def mark(self) -> None:
        if self.events[self.i] is None:
            self.events[self.i] = torch.cuda.Event()
        self.events[self.i].record()


def pack_upload(parts: list[tuple[str, np.ndarray]], staging: Staging, device):
    """Copy several small host arrays to the device in ONE transfer; returns views + bytes."""
    offs, off = [], 0
    for _, a in parts:
        off = (off + _ALIGN - 1) // _ALIGN * _ALIGN
        offs.append(off)
        off += a.nbytes
    total = max(off, _ALIGN)
    host = staging.get(total)
    hview = host.numpy()
    for (_, a), o in zip(parts, offs):
        b = np.ascontiguousarray(a).reshape(-1).view(np.uint8)
        hview[o:o + b.nbytes] = b
    device = torch.device(device)
    key = (device, total, tuple((name, a.dtype.str, a.shape) for name, a in parts))
    cached = staging.dev[staging.i]
    if cached is not None and cached[0] == key:
        dev, out = cached[1], cached[2]
    else:
        dev = torch.empty(total, dtype=torch.uint8, device=device)
        out = {}
        for (name, a), o in zip(parts, offs):
            out[name] = dev[o:o + a.nbytes].view(getattr(torch, a.dtype.name)).view(a.shape)
        staging.dev[staging.i] = (key, dev, out)
    dev.copy_(host, non_blocking=True)
    staging.mark()
    return dict(out), total
