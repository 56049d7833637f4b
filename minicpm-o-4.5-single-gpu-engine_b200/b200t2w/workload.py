"""Seeded synthetic workloads of the benchmark configurations.

No public dataset enters this path: the reference's Seed-TTS workload only shapes prompt lengths, and the uniform
ranges below stand in for it.  Every tensor is ~N(0,1) fp32, drawn on the CPU from ``torch.Generator().manual_seed``
in a fixed order, so every machine with this torch build draws the same values.

A stream is one request: a prompt of ``P`` frames and a chunk of ``T`` frames, solved as one packed ``[prompt | chunk]``
sequence of ``L = P + T`` frames.  ``spk`` is the speaker vector after the flow's speaker affine layer (``[mel]``), as
``FastDiT.solve`` takes it (``engine/runtime/dit_fast.py:436``).  ``cond`` is the prompt mel over the prompt frames
and zero over the chunk frames (the reference's setup solve conditions on the prompt mel, its chunk solves on zeros:
``engine/runtime/token2wav_batch.py:548-549,335``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    seed: int
    lengths: tuple  # ((P, T), ...) per stream

    @property
    def streams(self) -> int:
        return len(self.lengths)

    @property
    def chunk_frames(self) -> int:
        return sum(t for _, t in self.lengths)

    @property
    def packed_frames(self) -> int:
        return sum(p + t for p, t in self.lengths)


def uniform_streams(n: int, P: int, T: int) -> tuple:
    return tuple((P, T) for _ in range(n))


def ragged_streams(n: int, seed: int, p_range=(100, 500), t_range=(25, 100)) -> tuple:
    g = torch.Generator().manual_seed(seed)
    P = torch.randint(p_range[0], p_range[1] + 1, (n,), generator=g)
    T = torch.randint(t_range[0], t_range[1] + 1, (n,), generator=g)
    return tuple((int(p), int(t)) for p, t in zip(P, T))


C1 = Workload("c1_cpu_1x(200+50)", 0, uniform_streams(1, 200, 50))
C2 = Workload("c2_16x(300+50)", 1, uniform_streams(16, 300, 50))
C3 = Workload("c3_ragged64", 2, ragged_streams(64, 2))
C4 = Workload("c4_fp8_128x(300+50)", 1, uniform_streams(128, 300, 50))
C5 = Workload("c5_1024x(300+50)", 3, uniform_streams(1024, 300, 50))
TARGET = Workload("target_64x(300+50)", 1, uniform_streams(64, 300, 50))
CONFIGS = {w.name: w for w in (C1, C2, C3, C4, C5, TARGET)}


def make_streams(w: Workload, mel: int = 80, first: int = 0, count: int | None = None) -> list[dict]:
    """Streams ``first .. first + count`` of workload ``w`` (all of them by default).  Each stream's tensors come from
    its own generator seeded ``(w.seed, index)``, so any subset (a GPU shard, an oracle sample) draws the same values as
    the whole."""
    count = w.streams - first if count is None else count
    out = []
    for i in range(first, first + count):
        P, T = w.lengths[i]
        L = P + T
        g = torch.Generator().manual_seed(w.seed * 1_000_003 + i)
        x0 = torch.randn(mel, L, generator=g)
        mu = torch.randn(mel, L, generator=g)
        prompt = torch.randn(mel, P, generator=g)
        spk = torch.randn(mel, generator=g)
        cond = torch.cat([prompt, torch.zeros(mel, T)], dim=1)
        out.append({"x0": x0, "mu": mu, "cond": cond, "spk": spk, "P": P, "T": T, "index": i})
    return out
