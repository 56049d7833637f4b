"""CPU: the flow-encoder oracle against the golden fixtures made from the reference's own encoder driver code
(``tests/golden/make_encoder_golden.py``: ``_setup_encoder_batched``, ``_encoder`` with left-padded caches and masks,
``_flow_finish``'s trim).  The oracle's unpadded per-stream forward must reproduce every prompt setup and window to fp32
rounding; the seeded weights must be the ones the fixtures were made from."""

import copy
import dataclasses
import os

import pytest
import torch

from b200t2w.config import ENCODER, ENCODER_TINY, EncoderConfig
from oracle import encoder_oracle as eo
from tests.golden.make_encoder_golden import weights_digest


def rel(a, b):
    return float((a - b).norm() / b.norm())


def replay(flow, rec):
    """(oracle mu, fixture mu, label) for every prompt setup and window of a fixture, in call order."""
    out, sts = [], []
    for i, p in enumerate(rec["prompts"]):
        mu, st = eo.encode_prompt(flow, p["tokens"])
        sts.append(st)
        out.append((mu, p["mu"], f"prompt {i}"))
    for c, call in enumerate(rec["calls"]):
        for w in call["windows"]:
            st = sts[w["stream"]]
            if call["merged"] and w["final"]:  # a final riding in a steady call: as the same window alone, final
                mu = eo.encode_window(flow, copy.deepcopy(st), w["tokens"], True)
            else:
                mu = eo.encode_window(flow, st, w["tokens"], call["last"] or w["final"])
            out.append((mu, w["mu"], f"call {c} stream {w['stream']}"))
    return out


@pytest.mark.parametrize("name,cfg", [("encoder_tiny", ENCODER_TINY), ("encoder_reference", ENCODER)])
def test_encoder_oracle_matches_reference_driver(golden_dir, name, cfg):
    torch.set_num_threads(min(16, os.cpu_count() or 1))
    rec = torch.load(os.path.join(golden_dir, f"{name}.pt"))
    assert EncoderConfig(**rec["config"]) == cfg
    flow = eo.build_flow(cfg, seed=0)
    assert weights_digest(flow) == rec["weights_digest"], "seeded weights differ from the fixture's"
    got = replay(flow, rec)
    assert len(got) == len(rec["prompts"]) + sum(len(c["windows"]) for c in rec["calls"])
    for mu, ref, label in got:
        assert mu.shape == ref.shape, label
        assert rel(mu, ref) < 1e-5, label


def test_encoder_fixture_exercises_trim_merge_and_final(golden_dir):
    """The tiny fixture covers the cases the engine produces: the trim cutting caches, a final merged into a steady
    call, a final call, and streams of different cache lengths in one call."""
    rec = torch.load(os.path.join(golden_dir, "encoder_tiny.pt"))
    assert any(c["merged"] for c in rec["calls"]) and any(c["last"] for c in rec["calls"])
    flow = eo.build_flow(ENCODER_TINY, seed=0)
    sts = [eo.encode_prompt(flow, p["tokens"])[1] for p in rec["prompts"]]
    lens = [{st.att.shape[3] for st in sts}]
    trimmed = False
    for call in rec["calls"][:4]:
        for w in call["windows"]:
            st = sts[w["stream"]]
            before = st.att.shape[3]
            eo.encode_window(flow, st, w["tokens"], False)
            trimmed |= st.att.shape[3] < before + 2 * (len(w["tokens"]) - 3)
        lens.append({st.att.shape[3] for st in sts})
    assert trimmed
    assert all(len(s) > 1 for s in lens[:3])


def test_rel_shift_is_relative_position():
    """``rel_shift`` puts pe(L + i - j) at (query i, key j) for T queries after L cached keys."""
    T, L = 5, 7
    K = L + T
    x = torch.arange(2 * K - 1, dtype=torch.float32).repeat(1, 1, T, 1)  # column k holds k (position K - 1 - k)
    y = eo.RelPositionAttention.rel_shift(x)[0, 0]
    for i in range(T):
        for j in range(K):
            assert int(y[i, j]) == (K - 1) - (L + i - j)
