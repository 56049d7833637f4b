"""Generate the golden fixtures that pin the HiFT oracle (``oracle/hift_oracle.py``) to the reference's own vocoder
driver code.

Run in a container that has the reference checkout (read-only; never needed at test time)::

    python tests/golden/make_hift_golden.py --reference /path/to/reference

Per fixture: the restated vocoder (``hift_oracle.build_hift``) driven by the reference's ``BatchedToken2Wav._vocode``
(``engine/runtime/token2wav_batch.py:813-848``: windows grouped by mel / source-cache length, ``hift_forward`` with each
row's chunk seed, ``hift_noise``, ``hift_forward_noise``, ``_hift_decode``, ``istft_overlap_add``, ``fade_in_out``, the
cache update and the held-back tail; ``engine/models/token2wav.py:80-245``), in fp32 on the CPU, over calls that mix
first windows, steady windows and finals of several streams.  The oracle's per-stream restatement (``vocode_window``)
must reproduce every window's samples; the fixture stores the mels, the streams' noise seeds, the samples and the
weights' digest (weights are rebuilt from the seed).
"""

from __future__ import annotations

import argparse
import dataclasses
import hashlib
import os
import sys
from types import SimpleNamespace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "minicpm-o-4.5-single-gpu-engine_b200"))

from b200t2w.config import HIFT, HIFT_TINY  # noqa: E402
from oracle import hift_oracle as ho  # noqa: E402


def weights_digest(m) -> str:
    h = hashlib.sha256()
    sd = ho.state_dict_np(m)
    for k in sorted(sd):
        h.update(sd[k].tobytes())
    return h.hexdigest()[:32]


def rel(a, b) -> float:
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


# (stream, window mel frames, last) per call: first windows, steady windows, a final among steady ones, finals
CALLS = [
    [(0, 50, False), (1, 50, False), (2, 50, False)],
    [(0, 50, False), (1, 50, False), (2, 50, False)],
    [(0, 50, False), (1, 22, True), (2, 50, False)],
    [(0, 34, True), (2, 16, True)],
]


def make(cfg, name: str, seed: int) -> None:
    from engine.models.token2wav import StreamState
    from engine.runtime import token2wav_batch as tb

    hift = ho.build_hift(cfg, seed=0)
    bt = tb.BatchedToken2Wav.__new__(tb.BatchedToken2Wav)
    bt.hift, bt.hift_graphs, bt.hift_decode_tf32 = hift, None, False
    bt.t2w = SimpleNamespace(window=torch.from_numpy(np.hamming(2 * ho.SOURCE_CACHE)))
    g = torch.Generator().manual_seed(seed)
    noise_seeds = [int(x) for x in torch.randint(0, 1 << 30, (3,), generator=g)]
    sts = [StreamState(prompt=None, flow_cache={}, noise_seed=s,
                       hift_cache=dict(mel=torch.zeros(1, cfg.mel, 0), source=torch.zeros(1, 1, 0),
                                       speech=torch.zeros(1, 0))) for s in noise_seeds]
    ors = [ho.HiftStream(cfg.mel) for _ in sts]
    rec = {"config": dataclasses.asdict(cfg), "weights_digest": weights_digest(hift), "noise_seeds": noise_seeds,
           "calls": []}
    with torch.inference_mode():
        for call in CALLS:
            mels = [torch.randn(1, cfg.mel, T, generator=g) - 2.0 for _, T, _ in call]
            items = [(sts[i], None, last) for i, _, last in call]
            outs = bt._vocode(items, mels)
            got = []
            for (i, T, last), mel, out in zip(call, mels, outs):
                ref = torch.from_numpy(out)
                mine = ho.vocode_window(hift, ors[i], mel[0], ho.chunk_noise_seed(noise_seeds[i], ors[i].chunks), last)
                e = rel(mine, ref)
                assert mine.shape == ref.shape and e < 1e-5, (name, i, T, e)
                got.append({"stream": i, "last": last, "mel": mel[0].clone(), "samples": ref.clone()})
            print(f"{name} call {[(i, T, last) for i, T, last in call]}: oracle matches")
            rec["calls"].append(got)
    torch.save(rec, os.path.join(HERE, f"{name}.pt"))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    torch.set_num_threads(min(16, os.cpu_count() or 1))
    make(HIFT_TINY, "hift_tiny", seed=21)
    make(HIFT, "hift_reference", seed=22)


if __name__ == "__main__":
    main()
