"""Per-GPU stream scheduling: the reference worker's single-GPU loop (``engine/runtime/t2w_worker.py:302-621``,
``torch.cuda.set_device(0)`` at ``:804``) widened to every GPU of a node.

Token2Wav streams are independent: a solve touches only its own rows, caches and slots (``dit_fast.py:81-97``), so
there is no cross-GPU reduction and no collective.  A stream is placed on one GPU for its lifetime (its caches live
there) — the least-loaded GPU by outstanding packed frames at the time it opens — and each GPU's worker batches its own
streams' ready windows earliest-deadline-first (the reference's ``choose_windows`` policy, ``t2w_sched.py:100-105``).
``MultiGpuSolver`` drives one ``B200Solver`` per device from one host thread each (the C ABI releases the GIL).
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field


@dataclass
class GpuPlacement:
    """Sticky least-loaded placement of streams on ``n_gpus`` devices."""
    n_gpus: int
    load: list = field(default_factory=list)      # outstanding packed frames per device
    where: dict = field(default_factory=dict)     # stream id -> device

    def __post_init__(self):
        if self.n_gpus < 1:
            raise ValueError("need at least one GPU")
        if not self.load:
            self.load = [0] * self.n_gpus

    def open(self, stream_id, frames: int = 0) -> int:
        """Place a new stream (or return its device if already placed); ties go to the lowest device index."""
        if stream_id in self.where:
            return self.where[stream_id]
        dev = min(range(self.n_gpus), key=lambda d: (self.load[d], d))
        self.where[stream_id] = dev
        self.load[dev] += frames
        return dev

    def add(self, stream_id, frames: int) -> int:
        dev = self.where[stream_id]
        self.load[dev] += frames
        return dev

    def done(self, stream_id, frames: int) -> None:
        dev = self.where[stream_id]
        self.load[dev] = max(0, self.load[dev] - frames)

    def close(self, stream_id) -> None:
        self.where.pop(stream_id, None)


def shard_streams(lengths: list, n_gpus: int, contiguous: bool = False) -> list:
    """Partition stream indices over ``n_gpus``.  ``contiguous``: equal-count consecutive blocks (uniform workloads,
    config 5's 1024 / N); otherwise longest-first greedy on packed frames (P + T), which balances ragged batches."""
    n = len(lengths)
    if contiguous:
        per, extra = divmod(n, n_gpus)
        out, start = [], 0
        for g in range(n_gpus):
            cnt = per + (1 if g < extra else 0)
            out.append(list(range(start, start + cnt)))
            start += cnt
        return out
    order = sorted(range(n), key=lambda i: -(lengths[i][0] + lengths[i][1]))
    bins = [[] for _ in range(n_gpus)]
    load = [0] * n_gpus
    for i in order:
        g = min(range(n_gpus), key=lambda d: (load[d], d))
        bins[g].append(i)
        load[g] += lengths[i][0] + lengths[i][1]
    return [sorted(b) for b in bins]


def edf_windows(ready: list, max_rows: int | None = None) -> list:
    """``ready``: (deadline, key) per stream whose head window is ready; the keys to solve, earliest deadline first,
    at most ``max_rows`` (``t2w_sched.choose_windows`` semantics)."""
    order = sorted(ready, key=lambda x: x[0])
    if max_rows is not None:
        order = order[:max_rows]
    return [k for _, k in order]


class MultiGpuSolver:
    """One ``B200Solver`` per device; ``solve_streams`` shards a batch by ``shard_streams`` and runs every device's shard
    concurrently, returning per-stream results in input order and each device's event-timed milliseconds."""

    def __init__(self, cfg, weights: dict, devices: list, precision: str = "bf16"):
        import torch

        from .solver import B200Solver

        self.devices = [torch.device("cuda", d) if isinstance(d, int) else torch.device(d) for d in devices]
        self.solvers = []
        for dev in self.devices:
            with torch.cuda.device(dev):
                self.solvers.append(B200Solver(cfg, weights, precision=precision, device=dev))

    def solve_streams(self, streams: list, graph: bool = True) -> tuple:
        import torch

        parts = shard_streams([(s["P"], s["T"]) for s in streams], len(self.devices))
        results: list = [None] * len(streams)
        times = [0.0] * len(self.devices)
        errors: list = []

        def work(g: int) -> None:
            try:
                idx = parts[g]
                if not idx:
                    return
                dev = self.devices[g]
                with torch.cuda.device(dev):
                    st = torch.cuda.Stream(dev)
                    with torch.cuda.stream(st):
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record(st)
                        outs = self.solvers[g].solve_streams([streams[i] for i in idx], graph=graph)
                        e1.record(st)
                    st.synchronize()
                    times[g] = e0.elapsed_time(e1)
                for i, o in zip(idx, outs):
                    results[i] = o
            except Exception as e:  # a failed device fails only its own streams' call
                errors.append((g, e))

        threads = [threading.Thread(target=work, args=(g,)) for g in range(len(self.devices))]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise RuntimeError(f"device {errors[0][0]} failed: {errors[0][1]}") from errors[0][1]
        return results, times
