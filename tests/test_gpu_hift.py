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


@pytest.mark.parametrize("tf32", [False, True], ids=["fp32", "tf32"])
@pytest.mark.parametrize("name,cfg", [("hift_tiny", HIFT_TINY), ("hift_reference", HIFT)])
def test_vocode_vs_reference_driver_golden(golden_dir, name, cfg, tf32):
    """Strict fp32 (the reference's default) and the upsampling stages on TF32 tensor cores (its decode_tf32 option)."""
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


@pytest.mark.parametrize("tf32", [False, True], ids=["fp32", "tf32"])
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
