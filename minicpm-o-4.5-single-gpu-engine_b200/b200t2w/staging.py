"""Pinned host staging of solver inputs: a batch's host tensors are gathered into a pinned mirror of a static device
buffer and moved by one asynchronous copy, so the host never waits on a pageable copy (which synchronises the stream)
and can prepare the next call while the GPU runs this one."""

from __future__ import annotations

import torch


class HostStaging:
    """Pinned host mirrors of one static input buffer: a window's host tensors are concatenated into a mirror and moved
    by one asynchronous copy.  Two mirrors alternate; a mirror is rewritten once the copy that last read it is done."""

    def __init__(self, like: torch.Tensor):
        self.bufs = [torch.empty(like.shape, dtype=like.dtype).pin_memory() for _ in range(2)]
        self.events = [None, None]
        self.next = 0

    def copy(self, dst: torch.Tensor, src_host: torch.Tensor, stream) -> None:
        k = self.next
        self.next ^= 1
        if self.events[k] is not None:
            self.events[k].synchronize()
        self.bufs[k].copy_(src_host)
        dst.copy_(self.bufs[k], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self.events[k] = ev
