"""CPU: the HiFT vocoder oracle against the golden fixtures made from the reference's own vocoder driver
(``tests/golden/make_hift_golden.py``: ``BatchedToken2Wav._vocode`` -> ``hift_forward`` -> ``hift_forward_noise`` ->
``_hift_decode`` / ``istft_overlap_add``, the cross-fade, caches and held-back tail).  The oracle's per-stream
restatement must reproduce every window's samples to fp32 rounding, from weights rebuilt from the seed."""

import os

import pytest
import torch

from b200t2w.config import HIFT, HIFT_TINY, HiFTConfig
from oracle import hift_oracle as ho
from tests.golden.make_hift_golden import weights_digest


def rel(a, b):
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("name,cfg", [("hift_tiny", HIFT_TINY), ("hift_reference", HIFT)])
def test_hift_oracle_matches_reference_driver(golden_dir, name, cfg):
    torch.set_num_threads(min(16, os.cpu_count() or 1))
    rec = torch.load(os.path.join(golden_dir, f"{name}.pt"))
    got = {k: tuple(v) if isinstance(v, list) else v for k, v in rec["config"].items()}
    assert HiFTConfig(**got) == cfg
    hift = ho.build_hift(cfg, seed=0)
    assert weights_digest(hift) == rec["weights_digest"]
    sts = [ho.HiftStream(cfg.mel) for _ in rec["noise_seeds"]]
    n = 0
    for call in rec["calls"]:
        for w in call:
            st = sts[w["stream"]]
            out = ho.vocode_window(hift, st, w["mel"], ho.chunk_noise_seed(rec["noise_seeds"][w["stream"]], st.chunks),
                                   w["last"])
            assert out.shape == w["samples"].shape
            assert rel(out, w["samples"]) < 1e-5
            n += 1
    assert n == 11


def test_hift_fixture_is_not_degenerate(golden_dir):
    """Voiced and unvoiced frames both occur, and the waveform is neither silent nor clamped."""
    rec = torch.load(os.path.join(golden_dir, "hift_reference.pt"))
    hift = ho.build_hift(HIFT, seed=0)
    mel = torch.stack([w["mel"] for w in rec["calls"][1]])
    f0 = hift.f0_predictor(mel)
    voiced = float((f0 > HIFT.voiced_threshold).float().mean())
    assert 0.2 < voiced < 0.8, voiced
    s = torch.cat([w["samples"] for c in rec["calls"] for w in c])
    assert float(s.abs().max()) < HIFT.audio_limit and float(s.std()) > 1e-3
