"""GPU: the reference's own worker loop (``engine/runtime/t2w_worker.py`` ``WorkerLoop``) drives the B200 solver.

``b200t2w.worker.B200Token2Wav`` gives the loop the model calls it makes on ``BatchedToken2Wav`` (setup_many,
new_stream, release_stream / release_prompt, decode) with the DiT/CFM solve on ``B200FastDiT``.  The flow encoder and
the vocoder are outside this build, so the test passes stand-ins: the encoder maps each token to two fixed random mel
frames, the vocoder returns the window's mel as its samples.  Every window the loop emits must equal the CPU oracle's
streaming solve of that request (prompt setup, then its windows with the reference's trim, the last one not kept) within
the bf16 tolerance, and after the requests finish the worker's counters (``t2w_worker.py:827-834``) must show every
cache slot and conv-cache row returned.  The reference checkout comes from ``baseline/_ref`` (skipped without it); the
two-GPU placement half is skipped on a one-GPU box."""

import os
import sys
from types import SimpleNamespace

import pytest
import torch

from b200t2w.config import TINY
from b200t2w.fastdit import B200FastDiT
from b200t2w.solver import B200Solver, state_dict_from_module
from b200t2w.worker import B200Token2Wav, MultiGpuToken2Wav
from oracle import dit_oracle

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL = 1e-2
VOCAB = 64


def reference_loop():
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "engine")):
        pytest.skip("the reference checkout is not installed in baseline/_ref")
    if ref not in sys.path:
        sys.path.insert(0, ref)
    from engine.runtime.t2w_sched import Policy
    from engine.runtime.t2w_worker import WorkerLoop, setup_calls

    return WorkerLoop, Policy, setup_calls


def make_requests(seed: int):
    g = torch.Generator().manual_seed(seed)
    reqs = {}
    for seq, (ptok, wins) in {1: (60, (25, 25, 25, 10)), 2: (35, (25, 25, 7)), 3: (80, (25, 25, 25, 25, 12))}.items():
        reqs[seq] = {"prompt_tokens": torch.randint(0, VOCAB, (ptok,), generator=g).tolist(),
                     "mel": torch.randn(1, 2 * ptok, TINY.mel, generator=g), "spk": torch.randn(1, TINY.mel, generator=g),
                     "windows": [torch.randint(0, VOCAB, (n,), generator=g).tolist() for n in wins]}
    return reqs


def run_loop(bt, reqs):
    WorkerLoop, Policy, setup_calls = reference_loop()
    out = []
    feats = {seq: (r["prompt_tokens"], None, r["spk"], r["mel"], None) for seq, r in reqs.items()}
    loop = WorkerLoop(bt, out.append, lambda f: feats[f.seq],
                      lambda ready: setup_calls(ready, (512, 1024), {512: 8, 1024: 4}), Policy())
    for seq, r in reqs.items():
        loop.open(seq, seed=seq, fut=SimpleNamespace(seq=seq, done=lambda: True, result=lambda: None))
        for i, w in enumerate(r["windows"]):
            loop.window(seq, w, i == len(r["windows"]) - 1, i)
    for _ in range(100):
        loop.tick()
        if not loop.reqs:
            break
    assert not loop.reqs, "the loop did not finish every request"
    errors = [m for m in out if m[0] == "error"]
    assert not errors, errors
    audio = {}
    for m in out:
        if m[0] == "audio":
            audio.setdefault(m[1], []).append(m[3])
    return audio


def oracle_windows(model, table, r):
    mel = TINY.mel
    cache = dit_oracle.StreamCache(TINY, keep=r["mel"].shape[1])
    spk = r["spk"][0]
    enc = lambda toks: table[torch.tensor(toks)].reshape(-1, mel).t()  # noqa: E731
    outs = []
    for i, w in enumerate([r["prompt_tokens"]] + r["windows"]):
        mu = enc(w)
        T = mu.shape[1]
        x0 = model.rand_noise[0, :, cache.length:cache.length + T]
        cond = r["mel"][0].t() if i == 0 else None
        last = i == len(r["windows"])
        m = dit_oracle.solve_window(model, cache, x0, mu, spk, cond, keep_cache=not last)
        if i > 0:
            outs.append(m)
    return outs


def make_bt(model, table, device):
    fd = B200FastDiT(B200Solver(TINY, state_dict_from_module(model), device=device), model.rand_noise[0], n_slots=4096,
                     max_streams=8)
    enc = lambda toks: table[torch.tensor(toks)].reshape(-1, TINY.mel).t().to(fd.device)  # noqa: E731
    voc = lambda st, mel, last: mel.float().flatten().cpu().numpy()  # noqa: E731
    return fd, B200Token2Wav(fd, enc, voc, device_index=torch.device(device).index or 0)


def check(audio, reqs, model, table):
    for seq, r in reqs.items():
        ref = oracle_windows(model, table, r)
        got = audio[seq]
        assert len(got) == len(ref)
        for k, (a, b) in enumerate(zip(got, ref)):
            b = b.flatten()
            e = float((torch.from_numpy(a) - b).norm() / b.norm())
            print(f"request {seq} window {k} ({len(a) // TINY.mel} frames): rel-L2 vs oracle {e:.2e}")
            assert e < TOL


def test_reference_worker_loop_on_one_gpu():
    model = dit_oracle.build_model(TINY, seed=0, noise_frames=4096)
    table = torch.randn(VOCAB, 2, TINY.mel, generator=torch.Generator().manual_seed(5))
    fd, bt = make_bt(model, table, "cuda:0")
    free0 = len(fd.cnn_free)
    reqs = make_requests(3)
    audio = run_loop(bt, reqs)
    fd.solver.check()
    check(audio, reqs, model, table)
    # the worker's stats counters (t2w_worker.py:827-834) after every request finished
    assert fd.pool.in_use() - fd.scratch == 0
    assert len(fd.cnn_free) == free0
    n_windows = sum(len(r["windows"]) for r in reqs.values())
    assert 1 <= fd.counts["graph"] + fd.counts["eager"] <= n_windows + len(reqs)


def test_reference_worker_loop_across_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU on this box")
    model = dit_oracle.build_model(TINY, seed=0, noise_frames=4096)
    table = torch.randn(VOCAB, 2, TINY.mel, generator=torch.Generator().manual_seed(5))
    parts = [make_bt(model, table, f"cuda:{d}") for d in range(2)]
    mg = MultiGpuToken2Wav([bt for _, bt in parts])
    reqs = make_requests(4)
    audio = run_loop(mg, reqs)
    check(audio, reqs, model, table)
    assert mg.placement.load == [0, 0]
    assert {d for d in range(2) if parts[d][0].counts["eager"] + parts[d][0].counts["graph"]} == {0, 1}
    for fd, _ in parts:
        assert fd.pool.in_use() == 0


def test_reference_worker_loop_with_b200_flow_encoder():
    """The same loop with this build's flow encoder in place of the stand-in: prompts and windows are encoded by
    ``B200FlowEncoder`` (each request owns an encoder stream, copied from its prompt or adopted, advanced by every
    window, released with the request), then solved by ``B200FastDiT``.  Every window against the oracle's chain: the
    restated flow encoder's streaming forward (``encode_prompt`` / ``encode_window``) feeding the oracle's streaming solve;
    afterwards every encoder slot and stream is back."""
    from b200t2w.config import ENCODER_TINY
    from b200t2w.encoder import B200FlowEncoder
    from oracle import encoder_oracle as eo

    model = dit_oracle.build_model(TINY, seed=0, noise_frames=4096)
    flow = eo.build_flow(ENCODER_TINY, seed=0)
    fd = B200FastDiT(B200Solver(TINY, state_dict_from_module(model), device="cuda:0"), model.rand_noise[0], n_slots=4096,
                     max_streams=8)
    enc = B200FlowEncoder.from_flow(flow, device="cuda:0", max_frames=1024, n_slots1=4096, n_slots2=8192, n_streams=16,
                                    use_graphs=True)
    voc = lambda st, mel, last: mel.float().flatten().cpu().numpy()  # noqa: E731
    bt = B200Token2Wav(fd, enc, voc, device_index=0)
    g = torch.Generator().manual_seed(9)
    reqs = {}
    for seq, (ptok, wins) in {1: (60, (28, 28, 28, 10)), 2: (35, (28, 28, 7)), 3: (80, (28, 28, 28, 28, 12))}.items():
        reqs[seq] = {"prompt_tokens": torch.randint(0, VOCAB, (ptok,), generator=g).tolist(),
                     "mel": torch.randn(1, 2 * ptok, TINY.mel, generator=g), "spk": torch.randn(1, TINY.mel, generator=g),
                     "windows": [torch.randint(0, VOCAB, (n,), generator=g).tolist() for n in wins]}
    audio = run_loop(bt, reqs)
    fd.solver.check()
    enc.check()
    for seq, r in reqs.items():
        mu_p, est = eo.encode_prompt(flow, torch.tensor(r["prompt_tokens"]))
        cache = dit_oracle.StreamCache(TINY, keep=r["mel"].shape[1])
        spk = r["spk"][0]
        ref = []
        for i, w in enumerate([None] + r["windows"]):
            last = i == len(r["windows"])
            mu = mu_p if i == 0 else eo.encode_window(flow, est, torch.tensor(w), last)
            T = mu.shape[1]
            x0 = model.rand_noise[0, :, cache.length:cache.length + T]
            m = dit_oracle.solve_window(model, cache, x0, mu, spk, r["mel"][0].t() if i == 0 else None,
                                        keep_cache=not last)
            if i > 0:
                ref.append(m)
        got = audio[seq]
        assert len(got) == len(ref)
        for k, (a, b) in enumerate(zip(got, ref)):
            b = b.flatten()
            e = float((torch.from_numpy(a) - b).norm() / b.norm())
            print(f"request {seq} window {k} ({len(a) // TINY.mel} frames): rel-L2 vs oracle chain {e:.2e}")
            assert e < TOL
    assert enc.usage() == (0, 0, 0)
    assert fd.pool.in_use() - fd.scratch == 0


def test_reference_worker_loop_full_token2wav_chain():
    """Token2Wav end to end on this build: the reference's ``WorkerLoop`` drives ``B200Token2Wav`` with the B200 flow
    encoder, the B200 DiT solve and the B200 HiFT vocoder (TF32 upsampling stages).  Every window's samples against the
    oracle chain: the restated flow encoder's streaming forward -> the oracle's streaming solve -> the restated vocoder's
    ``vocode_window`` with the same source noise (drawn on the GPU from each chunk's seed, as the reference draws it);
    afterwards every encoder, solver and vocoder stream is back."""
    from b200t2w.config import ENCODER_TINY, HIFT_TINY
    from b200t2w.encoder import B200FlowEncoder
    from b200t2w.hift import B200HiFT, chunk_noise_seed
    from oracle import encoder_oracle as eo
    from oracle import hift_oracle as ho

    model = dit_oracle.build_model(TINY, seed=0, noise_frames=4096)
    flow = eo.build_flow(ENCODER_TINY, seed=0)
    hift = ho.build_hift(HIFT_TINY, seed=0)
    fd = B200FastDiT(B200Solver(TINY, state_dict_from_module(model), device="cuda:0"), model.rand_noise[0], n_slots=4096,
                     max_streams=8)
    enc = B200FlowEncoder.from_flow(flow, device="cuda:0", max_frames=1024, n_slots1=4096, n_slots2=8192, n_streams=16)
    voc = B200HiFT.from_module(hift, HIFT_TINY, device="cuda:0", max_frames=128, n_streams=16)
    bt = B200Token2Wav(fd, enc, voc, device_index=0)
    g = torch.Generator().manual_seed(17)
    reqs = {}
    for seq, (ptok, wins) in {1: (40, (28, 28, 10)), 2: (55, (28, 28, 28, 5))}.items():
        reqs[seq] = {"prompt_tokens": torch.randint(0, VOCAB, (ptok,), generator=g).tolist(),
                     "mel": torch.randn(1, 2 * ptok, TINY.mel, generator=g), "spk": torch.randn(1, TINY.mel, generator=g),
                     "windows": [torch.randint(0, VOCAB, (n,), generator=g).tolist() for n in wins]}
    audio = run_loop(bt, reqs)
    fd.solver.check()
    enc.check()
    voc.check()

    def gpu_noise(seed, n):
        gen = torch.Generator(device="cuda:0").manual_seed(int(seed))
        r = torch.rand(1, HIFT_TINY.harmonics + 1, device="cuda:0", generator=gen)
        z = torch.randn(1, HIFT_TINY.harmonics + 1, n, device="cuda:0", generator=gen)
        return r.cpu(), z.cpu().transpose(1, 2)

    for seq, r in reqs.items():
        mu_p, est = eo.encode_prompt(flow, torch.tensor(r["prompt_tokens"]))
        cache = dit_oracle.StreamCache(TINY, keep=r["mel"].shape[1])
        hst = ho.HiftStream(HIFT_TINY.mel)
        spk = r["spk"][0]
        x0 = model.rand_noise[0, :, cache.length:cache.length + mu_p.shape[1]]
        dit_oracle.solve_window(model, cache, x0, mu_p, spk, r["mel"][0].t(), keep_cache=True)
        got = audio[seq]
        assert len(got) == len(r["windows"])
        for k, w in enumerate(r["windows"]):
            last = k == len(r["windows"]) - 1
            mu = eo.encode_window(flow, est, torch.tensor(w), last)
            x0 = model.rand_noise[0, :, cache.length:cache.length + mu.shape[1]]
            mel = dit_oracle.solve_window(model, cache, x0, mu, spk, None, keep_cache=not last)
            ref = ho.vocode_window(hift, hst, mel, chunk_noise_seed(seq, k), last, noise_fn=gpu_noise)
            a = torch.from_numpy(got[k])
            e = float((a - ref).norm() / ref.norm())
            print(f"request {seq} window {k}: {a.numel()} samples, rel-L2 vs oracle chain {e:.2e}")
            # the chain's tolerance: the solve's bf16 mel (2e-3 of the oracle's) moves the vocoder's f0 and with it the
            # phase the source integrates, so the waveform moves by several times the mel's error (each stage alone is
            # checked at its own tolerance in its test)
            assert a.numel() == ref.numel() and e < 3e-2
    assert enc.usage() == (0, 0, 0)
    assert fd.pool.in_use() - fd.scratch == 0
