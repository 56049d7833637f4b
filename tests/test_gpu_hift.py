"""GPU: the HiFT vocoder (mel -> waveform) through the C ABI, strict fp32.

Against the golden fixtures made by the reference's own vocoder driver (``tests/golden/make_hift_golden.py``:
``BatchedToken2Wav._vocode`` over ``hift_forward_noise`` / ``_hift_decode`` / ``istft_overlap_add``, the cross-fade,
the caches and the held-back tail, on the restated HiFTGenerator) with the same seeded noise, and against the oracle on
ragged calls (every window its own frame count; first, steady and final windows mixed).  Tolerance: waveform rel-L2
<= 1e-2 (the reference's own bound for its vocoder against FP32); the kernels run in fp32, so the measured error is the
fp32 summation order amplified by the source's phase integration."""

import os

import pytest
import torch

from b200t2w import lib as L
from b200t2w.config import HIFT, HIFT_TINY
from b200t2w.hift import B200HiFT, chunk_noise_seed
from oracle import hift_oracle as ho

pytestmark = pytest.mark.gpu
TOL = 1e-2


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.fixture(scope="module", autouse=True)
def _dev():
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    assert L.load().t2w_device_ok(torch.cuda.current_device()) == 1


def oracle_noise(hift, seed, frames):
    r, nz = ho.hift_noise(hift, seed, 480 * frames)
    return r, nz.transpose(1, 2)


@pytest.mark.parametrize("tf32", [False, True, [1, 2, "0:src", "0:res"], ["2:res", "1:ups"]],
                         ids=["fp32", "tf32", "tf32_but_0ups", "tf32_2res_1ups"])
@pytest.mark.parametrize("name,cfg", [("hift_tiny", HIFT_TINY), ("hift_reference", HIFT)])
def test_vocode_vs_reference_driver_golden(golden_dir, name, cfg, tf32):
    """Strict fp32 (the reference's default), the upsampling stages on TF32 tensor cores (its decode_tf32 option), and
    two of its per-part lists (the parts left out on CUDA cores in fp32, their padding rows zeroed for the tensor-core
    parts that read them)."""
    rec = torch.load(os.path.join(golden_dir, f"{name}.pt"))
    hift = ho.build_hift(cfg, seed=0)
    voc = B200HiFT.from_module(hift, cfg, device="cuda", max_frames=128, n_streams=8, tf32=tf32)
    hs = [voc.new_stream(s) for s in rec["noise_seeds"]]
    chunks = [0, 0, 0]
    worst = 0.0
    for c, call in enumerate(rec["calls"]):
        noise = []
        for w in call:
            i = w["stream"]
            F = w["mel"].shape[1] + (0 if chunks[i] == 0 else 8)
            noise.append(oracle_noise(hift, chunk_noise_seed(rec["noise_seeds"][i], chunks[i]), F))
            chunks[i] += 1
        outs = voc.vocode([hs[w["stream"]] for w in call], [w["mel"] for w in call], [w["last"] for w in call],
                          noise=noise)
        for w, o in zip(call, outs):
            e = rel(o, w["samples"])
            worst = max(worst, e)
            print(f"{name} tf32={tf32} call {c} stream {w['stream']} ({w['mel'].shape[1]} frames, last={w['last']}): "
                  f"{o.numel()} samples, rel-L2 {e:.2e}")
            assert o.numel() == w["samples"].numel() and e < TOL
    print(f"{name} tf32={tf32}: worst window rel-L2 {worst:.2e}")
    voc.check()
    for h in hs:
        voc.release(h)


@pytest.mark.parametrize("tf32", [False, True, ["0:ups", "1:src", "2:res"]], ids=["fp32", "tf32", "tf32_mixed"])
def test_vocode_ragged_calls_vs_oracle(tf32):
    """Six streams, calls mixing first windows of different lengths, steady windows and finals, some streams skipping
    calls; every window against the oracle's per-stream ``vocode_window``."""
    torch.manual_seed(4)
    cfg = HIFT_TINY
    hift = ho.build_hift(cfg, seed=0)
    voc = B200HiFT.from_module(hift, cfg, device="cuda", max_frames=128, n_streams=8, tf32=tf32)
    seeds = [11, 22, 33, 44, 55, 66]
    hs = [voc.new_stream(s) for s in seeds]
    ors = [ho.HiftStream(cfg.mel) for _ in seeds]
    plan = [
        [(0, 50, False), (1, 16, False), (2, 30, False), (3, 50, False)],
        [(0, 50, False), (1, 50, False), (4, 40, False), (5, 12, True)],
        [(0, 50, True), (1, 50, False), (2, 50, False), (3, 7, True), (4, 50, False)],
        [(1, 21, True), (2, 50, True), (4, 3, True)],
    ]
    for c, call in enumerate(plan):
        mels = [torch.randn(cfg.mel, T) - 2.0 for _, T, _ in call]
        noise = []
        for (i, T, _) in call:
            F = T + (0 if ors[i].chunks == 0 else 8)
            noise.append(oracle_noise(hift, chunk_noise_seed(seeds[i], ors[i].chunks), F))
        outs = voc.vocode([hs[i] for i, _, _ in call], mels, [l for _, _, l in call], noise=noise)
        for (i, T, last), mel, o in zip(call, mels, outs):
            ref = ho.vocode_window(hift, ors[i], mel, chunk_noise_seed(seeds[i], ors[i].chunks), last)
            e = rel(o, ref)
            print(f"tf32={tf32} call {c} stream {i} T={T} last={last}: rel-L2 {e:.2e}")
            assert o.numel() == ref.numel() and e < TOL


def test_vocode_rejects_bad_calls():
    cfg = HIFT_TINY
    voc = B200HiFT.from_module(ho.build_hift(cfg, seed=0), cfg, device="cuda", max_frames=64, n_streams=2)
    h = voc.new_stream(1)
    with pytest.raises(L.T2WError):  # more frames than max_frames
        voc.vocode([h], [torch.zeros(cfg.mel, 80)], [False])
    with pytest.raises(L.T2WError):  # a first window that is not final needs 8 frames
        voc.vocode([h], [torch.zeros(cfg.mel, 5)], [False])
    with pytest.raises(L.T2WError):  # the same stream twice
        voc.vocode([h, h], [torch.zeros(cfg.mel, 20)] * 2, [False, False])


def test_seeded_noise_matches_reference_draws():
    """Without ``noise=`` every window's source noise is the reference's ``hift_noise`` on the vocoder's device: a CUDA
    generator seeded with the chunk seed, ``rand(1, dim)`` then ``randn(1, dim, 480 F)`` (engine/models/token2wav.py:
    112-121).  The same windows vocoded with those draws passed explicitly give bit-identical samples."""
    cfg = HIFT_TINY
    hift = ho.build_hift(cfg, seed=0)
    dim = cfg.harmonics + 1
    a = B200HiFT.from_module(hift, cfg, device="cuda", max_frames=64, n_streams=4)
    b = B200HiFT.from_module(hift, cfg, device="cuda", max_frames=64, n_streams=4)
    seeds = [7, 123456789, 2 ** 40 + 3]
    ha = [a.new_stream(s) for s in seeds]
    hb = [b.new_stream(s) for s in seeds]
    g = torch.Generator().manual_seed(9)
    for c, (Ts, lasts) in enumerate((([50, 20, 50], [False, False, True]), ([50, 50], [False, True]))):
        n = len(Ts)
        mels = [torch.randn(cfg.mel, T, generator=g) - 2.0 for T in Ts]
        noise = []
        for i in range(n):
            F = Ts[i] + (8 if c else 0)
            gen = torch.Generator(device="cuda").manual_seed(chunk_noise_seed(seeds[i], c))
            noise.append((torch.rand(1, dim, device="cuda", generator=gen),
                          torch.randn(1, dim, 480 * F, device="cuda", generator=gen)))
        oa = a.vocode(ha[:n], mels, lasts)
        ob = b.vocode(hb[:n], mels, lasts, noise=noise)
        for x, y in zip(oa, ob):
            assert x.numel() == y.numel() and torch.equal(x, y)
    a.close()
    b.close()


def test_tf32_mode_source_is_fp32_accurate():
    """With ``tf32`` the f0 predictor runs on the tensor cores in split form (3xTF32), where the reference keeps fp32:
    the harmonic source it drives (f0 -> phase -> sines) against the strict-fp32 build's, both windows of a stream (the
    second with its cached mel frames).  The source integrates f0 into a phase of hundreds of radians per window, so
    it magnifies f0 differences: the split layers' 1.2e-5 per layer (``tests/test_gpu_tconv.py``, against plain TF32's
    8e-4) shows here as ~4e-4; bound 1e-3."""
    cfg = HIFT
    hift = ho.build_hift(cfg, seed=0)
    vs = {t: B200HiFT.from_module(hift, cfg, device="cuda", max_frames=64, n_streams=4, tf32=t) for t in (False, True)}
    hs = {t: [v.new_stream(s) for s in (3, 4)] for t, v in vs.items()}
    g = torch.Generator().manual_seed(21)
    for c in range(2):
        mels = [torch.randn(cfg.mel, 50, generator=g) - 2.0 for _ in range(2)]
        F = 50 + (8 if c else 0)
        noise = [oracle_noise(hift, chunk_noise_seed(s, c), F) for s in (3, 4)]
        src = {}
        for t, v in vs.items():
            src[t] = torch.empty(2 * 480 * F, device="cuda")
            v.vocode(hs[t], mels, [False, False], noise=noise, source=src[t])
        e = rel(src[True], src[False])
        print(f"window {c}: source rel-L2 tf32 vs strict {e:.2e}")
        assert e < 1e-3


@pytest.mark.parametrize("name,cfg", [("hift_tiny", HIFT_TINY), ("hift_reference", HIFT)])
def test_split_fp32_mode_vs_reference_driver_golden(golden_dir, name, cfg):
    """``split_fp32``: every convolution on the tensor cores in split form (3xTF32), the reference's strict-fp32
    numerics (its default) at tensor-core speed.  Against the reference driver's fp32 golden fixtures, calls mixing
    first, steady and final windows: measured 1.4e-5 (tiny) / 2.1e-4 - 3.6e-4 (reference config, depending on the
    convolutions' accumulation order), bound 5e-4 — against the TF32 mode's 8e-4 / 1.6e-3 and the CUDA-core strict
    mode's 3e-6 / 1e-5; most of it is the f0 predictor's split-form rounding (1e-5 a layer) carried into the source's
    phase."""
    rec = torch.load(os.path.join(golden_dir, f"{name}.pt"))
    hift = ho.build_hift(cfg, seed=0)
    voc = B200HiFT.from_module(hift, cfg, device="cuda", max_frames=128, n_streams=8, split_fp32=True)
    hs = [voc.new_stream(s) for s in rec["noise_seeds"]]
    chunks = [0, 0, 0]
    worst = 0.0
    for call in rec["calls"]:
        noise = []
        for w in call:
            i = w["stream"]
            F = w["mel"].shape[1] + (0 if chunks[i] == 0 else 8)
            noise.append(oracle_noise(hift, chunk_noise_seed(rec["noise_seeds"][i], chunks[i]), F))
            chunks[i] += 1
        outs = voc.vocode([hs[w["stream"]] for w in call], [w["mel"] for w in call], [w["last"] for w in call],
                          noise=noise)
        for w, o in zip(call, outs):
            e = rel(o, w["samples"])
            worst = max(worst, e)
            assert o.numel() == w["samples"].numel() and e < 5e-4, e
    print(f"{name} split_fp32: worst window rel-L2 {worst:.2e}")
    voc.check()


@pytest.mark.parametrize("split_fp32", [False, True], ids=["tf32", "split_fp32"])
def test_graph_replay_equals_eager(split_fp32):
    """``use_graphs`` (the reference's ``t2w_graphs`` / ``HiFTGraphs``): a stream's first windows, steady windows that
    repeat a call structure (captured on its second sight, replayed after) and finals, bit-identical to the eager
    vocoder's samples with the same seeded noise; the counters show the captures and replays."""
    cfg = HIFT_TINY
    hift = ho.build_hift(cfg, seed=0)
    kw = dict(device="cuda", max_frames=64, n_streams=8, split_fp32=split_fp32)
    vg = B200HiFT.from_module(hift, cfg, use_graphs=True, **kw)
    ve = B200HiFT.from_module(hift, cfg, **kw)
    seeds = [5, 6, 7]
    hg = [vg.new_stream(s) for s in seeds]
    he = [ve.new_stream(s) for s in seeds]
    g = torch.Generator().manual_seed(8)
    plan = [[50, 50, 50]] + [[50, 50, 50]] * 4 + [[12, 30, 7]]
    for c, Ts in enumerate(plan):
        last = c == len(plan) - 1
        mels = [torch.randn(cfg.mel, T, generator=g) - 2.0 for T in Ts]
        og = vg.vocode(hg, mels, [last] * 3)
        oe = ve.vocode(he, mels, [last] * 3)
        for a, b in zip(og, oe):
            assert a.numel() == b.numel() and torch.equal(a, b), c
    cnt = vg.counts
    print(f"split_fp32={split_fp32}: {cnt}")
    assert cnt["captures"] >= 1 and cnt["replays"] >= 3
    assert ve.counts["replays"] == 0
    vg.check()


@pytest.mark.parametrize("split_fp32", [False, True], ids=["tf32", "split_fp32"])
def test_caller_stream_equals_default_stream(split_fp32):
    """A call forks its independent branches (the f0 predictor, source and STFT, every stage's source branch, two of
    each stage's three ResBlocks, the seeded draws) onto streams of the vocoder's own and joins them back: called from
    a non-blocking stream of the caller's, with back-to-back calls and no synchronisation between them, the samples
    equal the default-stream calls' bit for bit."""
    cfg = HIFT_TINY
    hift = ho.build_hift(cfg, seed=0)
    kw = dict(device="cuda", max_frames=64, n_streams=8, split_fp32=split_fp32)
    va = B200HiFT.from_module(hift, cfg, **kw)
    vb = B200HiFT.from_module(hift, cfg, **kw)
    seeds = [3, 4, 9]
    ha = [va.new_stream(s) for s in seeds]
    hb = [vb.new_stream(s) for s in seeds]
    g = torch.Generator().manual_seed(12)
    plan = [[50, 50, 50], [50, 50, 50], [50, 50, 50], [20, 45, 9]]
    calls = [[torch.randn(cfg.mel, T, generator=g) - 2.0 for T in Ts] for Ts in plan]
    ref = [va.vocode(ha, m, [c == len(plan) - 1] * 3) for c, m in enumerate(calls)]
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        got = [vb.vocode(hb, m, [c == len(plan) - 1] * 3) for c, m in enumerate(calls)]
    side.synchronize()
    for c, (ra, rb) in enumerate(zip(ref, got)):
        for a, b in zip(ra, rb):
            assert a.numel() == b.numel() and torch.equal(a, b), c
    va.check()
    vb.check()
