"""CPU: the oracle against the golden fixtures made from the reference's own solver code (tests/golden/make_golden.py).

The fixtures hold the reference driver's outputs (``BatchedToken2Wav._solve``: prompt setup, then the chunk against its
caches) run on the restated estimator modules; the oracle's packed ``[prompt | chunk]`` solve must reproduce them to
fp32 rounding.  Digests check that the seeded weights and inputs are the ones the fixtures were made from.
"""

import os

import pytest
import torch

from b200t2w.config import REFERENCE, TINY, DiTConfig, t_schedule
from b200t2w.workload import C1, C2, C3, make_streams
from oracle import dit_oracle
from tests.golden.make_golden import digest, weights_digest


def rel(a, b):
    return float((a - b).norm() / b.norm())


def _check_fixture(path, cfg, streams_from):
    rec = torch.load(path)
    assert DiTConfig(**rec["config"]) == cfg
    model = dit_oracle.build_model(cfg, seed=0, noise_frames=max(s["P"] + s["T"] for s in rec["streams"]) + 8)
    assert weights_digest(model) == rec["weights_digest"], "seeded weights differ from the fixture's"
    for s, g in zip(streams_from(rec), rec["streams"]):
        assert digest(s["x0"], s["mu"], s["cond"], s["spk"]) == g["inputs_digest"]
        out = dit_oracle.solve_packed(model, s["x0"], s["mu"], s["cond"], s["spk"], s["P"], s["T"])
        assert rel(out[:, :s["P"]], g["ref_prompt_mel"]) < 1e-5
        assert rel(out[:, s["P"]:], g["ref_chunk_mel"]) < 1e-5


def test_oracle_tiny_ragged_matches_reference_driver(golden_dir):
    _check_fixture(os.path.join(golden_dir, "tiny_ragged.pt"), TINY, lambda rec: rec["streams"])


def test_oracle_c1_full_size_matches_reference_driver(golden_dir):
    torch.set_num_threads(os.cpu_count() or 1)
    _check_fixture(os.path.join(golden_dir, "c1_reference.pt"), REFERENCE, lambda rec: make_streams(C1))


def test_oracle_steady_windows_match_reference_driver(golden_dir):
    """Steady state: the prompt setup then runs of windows against the caches, with the reference's trim (first P plus
    the last 100 keys) and final flushes that leave the caches untouched."""
    rec = torch.load(os.path.join(golden_dir, "steady_tiny.pt"))
    assert DiTConfig(**rec["config"]) == TINY
    model = dit_oracle.build_model(TINY, seed=0, noise_frames=2048)
    assert weights_digest(model) == rec["weights_digest"]
    trimmed = False
    for s in rec["streams"]:
        cache = dit_oracle.StreamCache(TINY, keep=s["P"])
        for w in s["windows"]:
            assert torch.equal(w["x0"], model.rand_noise[0, :, cache.length:cache.length + w["T"]])
            before = cache.length
            mel = dit_oracle.solve_window(model, cache, w["x0"], w["mu"], s["spk"], w["cond"], keep_cache=w["keep"])
            assert rel(mel, w["ref_mel"]) < 1e-5
            assert cache.length == w["cache_len_after"]
            trimmed |= w["keep"] and cache.length < before + w["T"]
    assert trimmed, "the fixture must exercise the trim"


def test_block_causal_mask():
    m = dit_oracle.block_causal_mask(3, 2)
    assert m.shape == (5, 5)
    assert m[:3, :3].all() and not m[:3, 3:].any() and m[3:].all()
    assert dit_oracle.block_causal_mask(4, 0).all()


def test_t_schedule_recurrence():
    ts, dts = t_schedule(10)
    assert ts[0] == 0.0 and len(ts) == len(dts) == 10
    assert all(b > a for a, b in zip(ts, ts[1:]))
    assert abs(ts[-1] + dts[-1] - 1.0) < 1e-6


def test_workload_subsets_are_stable():
    a = make_streams(C2, first=3, count=2)
    b = make_streams(C2)[3:5]
    for x, y in zip(a, b):
        assert torch.equal(x["x0"], y["x0"]) and torch.equal(x["spk"], y["spk"]) and x["P"] == y["P"]
    assert C3.streams == 64 and all(100 <= p <= 500 and 25 <= t <= 100 for p, t in C3.lengths)
    s = make_streams(C1)[0]
    assert s["cond"][:, s["P"]:].abs().sum() == 0


def test_uncond_row_ignores_conditioning():
    """The CFG uncond row zeroes mu / spk / cond (token2wav_batch.py:672-674): with w = 0 the solve is the cond row's
    plain Euler solve; changing the conditioning changes the result."""
    cfg = TINY
    model = dit_oracle.build_model(cfg, seed=0)
    s = make_streams(C1, mel=cfg.mel)[0]
    s = {k: (v[:, :40] if torch.is_tensor(v) and v.dim() == 2 else v) for k, v in s.items()}
    s["cond"][:, 30:] = 0
    a = dit_oracle.solve_packed(model, s["x0"], s["mu"], s["cond"], s["spk"], 30, 10)
    b = dit_oracle.solve_packed(model, s["x0"], s["mu"] * 0.5, s["cond"], s["spk"], 30, 10)
    assert rel(a, b) > 1e-3


@pytest.mark.parametrize("P,T", [(7, 5), (1, 1), (12, 0)])
def test_packed_equals_chunk_with_prompt_only_keys(P, T):
    """Prompt frames of a packed solve equal a solve of the prompt alone (prompt queries never see chunk keys and the
    convolutions are causal)."""
    cfg = TINY
    model = dit_oracle.build_model(cfg, seed=1)
    g = torch.Generator().manual_seed(P * 100 + T)
    x0, mu, cond = (torch.randn(cfg.mel, P + T, generator=g) for _ in range(3))
    spk = torch.randn(cfg.mel, generator=g)
    full = dit_oracle.solve_packed(model, x0, mu, cond, spk, P, T)
    alone = dit_oracle.solve_packed(model, x0[:, :P], mu[:, :P], cond[:, :P], spk, P, 0)
    assert rel(full[:, :P], alone) < 1e-5
