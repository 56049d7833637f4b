"""CPU: the multi-GPU worker surface (``b200t2w.worker.MultiGpuToken2Wav``) over fake per-device models.

Requests are placed on the least-loaded device when their prompts are set up and stay there; a decode call's windows
are split by device and the samples come back in the call's order; releasing a stream frees its device's load; a
failing device fails the call and leaves nothing placed.  When the reference checkout is installed in
``baseline/_ref``, the reference's own ``WorkerLoop`` drives the surface end to end."""

import os
import sys
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from b200t2w.worker import B200Prompt, B200Stream, MultiGpuToken2Wav

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class FakeDevice:
    """One device's model: records calls; samples encode (device, window length, last)."""

    def __init__(self, d, fail=False):
        self.d, self.fail, self.calls, self.live = d, fail, [], 0

    def setup_many(self, feats):
        if self.fail:
            raise RuntimeError(f"device {self.d} failed")
        self.calls.append(("setup", len(feats)))
        self.live += len(feats)
        return [B200Prompt(object(), torch.zeros(1, 4), int(f[3].shape[1]), self.d) for f in feats]

    def new_stream(self, prompt, noise_seed=0, adopt=False):
        return B200Stream(prompt.cache, prompt.spk, noise_seed, 0, self.d)

    def release_stream(self, st):
        self.live -= 1

    def release_prompt(self, p):
        self.live -= 1

    def decode(self, items):
        self.calls.append(("decode", len(items)))
        return [np.full(len(tok), 100 * self.d + (1 if last else 0), np.float32) for _, tok, last in items]


def feats(frames):
    return ([1, 2, 3], None, torch.zeros(1, 4), torch.zeros(1, frames, 4), None)


def test_least_loaded_sticky_placement_and_ordered_results():
    devs = [FakeDevice(0), FakeDevice(1)]
    mg = MultiGpuToken2Wav(devs)
    ps = mg.setup_many([feats(300), feats(100), feats(150)])
    assert [p.device for p in ps] == [0, 1, 1]  # 300 on 0; 100 on 1; 150 on 1 (load 100 < 300)
    sts = [mg.new_stream(p, noise_seed=i, adopt=True) for i, p in enumerate(ps)]
    out = mg.decode([(sts[2], [0] * 5, False), (sts[0], [0] * 7, True), (sts[1], [0] * 3, False)])
    assert [len(o) for o in out] == [5, 7, 3]
    assert [float(o[0]) for o in out] == [100.0, 1.0, 100.0]
    assert ("decode", 1) in devs[0].calls and ("decode", 2) in devs[1].calls
    assert mg.placement.load == [300, 250]
    mg.release_stream(sts[0])
    assert mg.placement.load == [0, 250] and devs[0].live == 0
    p = mg.setup_many([feats(50)])[0]
    assert p.device == 0  # device 0 is now the least loaded


def test_failed_device_fails_the_call_and_leaves_nothing_placed():
    devs = [FakeDevice(0), FakeDevice(1, fail=True)]
    mg = MultiGpuToken2Wav(devs)
    with pytest.raises(RuntimeError):
        mg.setup_many([feats(100), feats(100)])
    assert mg.placement.load == [0, 0] and not mg.placement.where
    assert devs[0].live == 0  # the prompt set up on the healthy device went back


def test_reference_worker_loop_drives_the_surface():
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "engine")):
        pytest.skip("the reference checkout is not installed in baseline/_ref")
    sys.path.insert(0, ref)
    from engine.runtime.t2w_sched import Policy
    from engine.runtime.t2w_worker import WorkerLoop, setup_calls

    devs = [FakeDevice(0), FakeDevice(1)]
    mg = MultiGpuToken2Wav(devs)
    out = []
    fut = SimpleNamespace(done=lambda: True, result=lambda: None)
    frames = {1: 300, 2: 120, 3: 200}
    loop = WorkerLoop(mg, out.append, lambda f: feats(frames[f.seq]),
                      lambda ready: setup_calls(ready, (512, 1024), {512: 8, 1024: 4}), Policy())
    for seq in frames:
        loop.open(seq, seed=seq, fut=SimpleNamespace(seq=seq, done=fut.done, result=fut.result))
        loop.window(seq, [0] * 28, False, 0)
        loop.window(seq, [0] * 28, True, 1)
    for _ in range(20):
        loop.tick()
        if not loop.reqs:
            break
    assert not loop.reqs
    done = {m[1] for m in out if m[0] == "done"}
    assert done == set(frames)
    audio = [m for m in out if m[0] == "audio"]
    assert len(audio) == 6 and all(len(m[3]) == 28 for m in audio)
    assert mg.placement.load == [0, 0] and devs[0].live == 0 and devs[1].live == 0
