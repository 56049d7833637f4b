"""The Token2Wav worker's model surface on the B200 solver, on one GPU or spread over several.

The reference worker (``engine/runtime/t2w_worker.py`` ``WorkerLoop``, ``:302-621``) drives its model through five
calls of ``BatchedToken2Wav`` (``engine/runtime/token2wav_batch.py:221-309,508-554``): ``setup_many`` (prompt setups),
``new_stream`` (a request's stream from its prompt, adopting the prompt's caches), ``release_stream`` /
``release_prompt``, and ``decode`` (one window per request -> samples).  ``B200Token2Wav`` provides those calls with the
DiT/CFM solve on ``B200FastDiT``: a setup solves the prompt's frames with the prompt mel as condition and keeps its keys
(trim length = the prompt's mel frames, as ``setup_many`` sets ``c.keep``), a window solves against the stream's caches
and keeps its keys unless it is the stream's last (``keep = not last``, as ``_flow_encode`` sets it).  The flow encoder
(tokens -> ``mu``) is either this build's ``B200FlowEncoder`` — then every prompt and request owns an encoder stream
(its conformer caches), set up, copied or adopted, advanced and released with the DiT caches, and a decode call encodes
all its windows in one call, as ``_flow_encode`` does — or any callable ``tokens -> mu``.  The HiFT vocoder (mel ->
samples) is likewise this build's ``B200HiFT`` — every request owns a vocoder stream (its mel / source / speech
caches and its noise seed), and a decode call vocodes all its windows in one call, as ``_vocode`` does — or a callable
``(stream, mel, last) -> samples``.

``MultiGpuToken2Wav`` is the same surface over one ``B200Token2Wav`` per GPU, in place of the reference worker's single
device (``torch.cuda.set_device(0)``, ``t2w_worker.py:804``): a request is placed on the least-loaded GPU when its prompt
is set up (``scheduler.GpuPlacement``, sticky: its caches live there), a decode call's windows are split by device and
each device's part runs in a thread of its own, and the samples come back in the call's order.  There is no
collective: requests never cross GPUs.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass

import torch

from .scheduler import GpuPlacement


@dataclass
class B200Prompt:
    """A set-up prompt: its estimator caches (until a stream adopts them), speaker vector and mel frames, and its flow
    encoder stream when the encoder is a ``B200FlowEncoder``."""
    cache: object
    spk: torch.Tensor  # [1, mel] after the flow's speaker affine layer
    frames: int
    device: int = 0
    enc: int | None = None


@dataclass
class B200Stream:
    """One request's stream: its caches, speaker vector, and the windows decoded so far."""
    cache: object
    spk: torch.Tensor
    noise_seed: int = 0
    chunks: int = 0
    device: int = 0
    enc: int | None = None
    voc: int | None = None


class B200Token2Wav:
    """``BatchedToken2Wav``'s worker-facing calls on one GPU.

    ``fast``: a ``B200FastDiT``.  ``encode(tokens) -> mu [mel, frames]``: the flow encoder of a window or a prompt's
    tokens.  ``vocode(stream, mel [mel, T] fp32, last) -> samples``: the vocoder of one window's mel.  ``features`` of a
    setup are the reference's tuple ``(tokens, _, spk [1, mel] post-affine, prompt mel [1, frames, mel], _)``; the
    worker's ``setup_calls`` reads ``feats[3].shape[1]``."""

    def __init__(self, fast, encode, vocode, device_index: int = 0):
        from .encoder import B200FlowEncoder
        from .hift import B200HiFT

        self.fast, self.encode, self.vocode, self.device_index = fast, encode, vocode, device_index
        self.flow = encode if isinstance(encode, B200FlowEncoder) else None
        self.hift = vocode if isinstance(vocode, B200HiFT) else None
        self.dev = fast.device

    @staticmethod
    def _tokens(t) -> list:
        return [int(x) for x in (t.flatten().tolist() if isinstance(t, torch.Tensor) else t)]

    def setup_many(self, feats_list: list) -> list:
        caches = [self.fast.new_cache() for _ in feats_list]
        handles = []
        try:
            if self.flow is not None:  # every prompt through a new encoder stream, one call
                handles, enc_mus = self.flow.setup([self._tokens(f[0]) for f in feats_list])
            mus, conds, spks = [], [], []
            for i, (c, f) in enumerate(zip(caches, feats_list)):
                mel = f[3][0].t()  # [mel, frames]
                c.keep = int(mel.shape[1])  # the trim length: the prompt's mel frames (token2wav_batch.py:544)
                mu = enc_mus[i] if self.flow is not None else self.encode(f[0])
                if int(mu.shape[1]) != int(mel.shape[1]):
                    raise ValueError(f"prompt: the encoder gave {mu.shape[1]} frames for a {mel.shape[1]}-frame mel")
                mus.append(mu)
                conds.append(mel)
                spks.append(f[2].reshape(1, -1))
            spk = torch.cat(spks).to(self.dev, torch.float32)
            self.fast.solve(caches, mus, spk, conds, [True] * len(caches))
        except Exception:
            for c in caches:
                self.fast.release(c)
            for h in handles:
                self.flow.release(h)
            raise
        return [B200Prompt(c, spk[i:i + 1], int(m.shape[1]), self.device_index, handles[i] if handles else None)
                for i, (c, m) in enumerate(zip(caches, conds))]

    def new_stream(self, prompt: B200Prompt, noise_seed: int = 0, adopt: bool = False) -> B200Stream:
        if adopt:  # the prompt is used once: its caches become the stream's
            cache, prompt.cache = prompt.cache, None
            enc, prompt.enc = prompt.enc, None
        else:
            cache = self.fast.clone(prompt.cache)
            enc = self.flow.clone(prompt.enc) if prompt.enc is not None else None
        voc = self.hift.new_stream(noise_seed) if self.hift is not None else None
        return B200Stream(cache, prompt.spk, noise_seed, 0, self.device_index, enc, voc)

    def release_stream(self, st: B200Stream) -> None:
        if st is not None and st.cache is not None:
            self.fast.release(st.cache)
            st.cache = None
        if st is not None and st.enc is not None:
            self.flow.release(st.enc)
            st.enc = None
        if st is not None and st.voc is not None:
            self.hift.release(st.voc)
            st.voc = None

    def release_prompt(self, p: B200Prompt) -> None:
        if p is not None and p.cache is not None:
            self.fast.release(p.cache)
            p.cache = None
        if p is not None and p.enc is not None:
            self.flow.release(p.enc)
            p.enc = None

    def decode(self, items: list) -> list:
        """``items[i] = (stream, window tokens, last)`` -> samples per item (one encoder call and one solve for every
        window of the call)."""
        if not items:
            return []
        sts = [it[0] for it in items]
        if self.flow is not None:
            mus = self.flow.encode([st.enc for st in sts], [self._tokens(it[1]) for it in items],
                                   [bool(it[2]) for it in items])
        else:
            mus = [self.encode(it[1]) for it in items]
        spk = torch.cat([st.spk for st in sts])
        mels = self.fast.solve([st.cache for st in sts], mus, spk, None, [not bool(it[2]) for it in items])
        if self.hift is not None:  # every window's samples from one vocoder call and one device-to-host copy
            out = self.hift.vocode_numpy([st.voc for st in sts], mels, [bool(it[2]) for it in items])
            for st in sts:
                st.chunks += 1
            return out
        out = []
        for st, mel, it in zip(sts, mels, items):
            out.append(self.vocode(st, mel, bool(it[2])))
            st.chunks += 1
        return out


class MultiGpuToken2Wav:
    """The worker surface over one ``B200Token2Wav`` per GPU (``parts``), requests placed by ``GpuPlacement``."""

    def __init__(self, parts: list):
        if not parts:
            raise ValueError("need at least one device")
        self.parts = parts
        self.placement = GpuPlacement(len(parts))
        self._frames: dict = {}  # placement key -> the frames its request added to its device's load
        self._next_id = 0
        self._lock = threading.Lock()

    def setup_many(self, feats_list: list) -> list:
        # each new request on the least-loaded device at this moment (load = packed frames of its open requests)
        where = []
        with self._lock:
            for f in feats_list:
                key = ("req", self._next_id)
                self._next_id += 1
                self._frames[key] = int(f[3].shape[1])
                where.append((key, self.placement.open(key, self._frames[key])))
        groups: dict = {}
        for i, (_, d) in enumerate(where):
            groups.setdefault(d, []).append(i)
        out: list = [None] * len(feats_list)

        def run(d, idx):
            ps = self.parts[d].setup_many([feats_list[i] for i in idx])
            for i, p in zip(idx, ps):
                p.device = d
                p.place_key = where[i][0]
                out[i] = p

        try:
            self._each(groups, run)
        except Exception:  # the call fails as a whole: set-up prompts of the other devices go back, nothing stays placed
            for i, (key, _) in enumerate(where):
                if out[i] is not None:
                    self.parts[out[i].device].release_prompt(out[i])
                self._unplace(key)
            raise
        return out

    def new_stream(self, prompt, noise_seed: int = 0, adopt: bool = False):
        st = self.parts[prompt.device].new_stream(prompt, noise_seed=noise_seed, adopt=adopt)
        st.device = prompt.device
        st.place_key = getattr(prompt, "place_key", None)
        prompt.adopted = adopt  # an adopted prompt's placement now belongs to its stream
        return st

    def _unplace(self, key) -> None:
        if key is None:
            return
        with self._lock:
            if key in self.placement.where:
                self.placement.done(key, self._frames.pop(key, 0))
                self.placement.close(key)

    def release_stream(self, st) -> None:
        if st is None:
            return
        self.parts[st.device].release_stream(st)
        self._unplace(getattr(st, "place_key", None))

    def release_prompt(self, p) -> None:
        if p is None:
            return
        self.parts[p.device].release_prompt(p)
        if p.cache is None and getattr(p, "adopted", False):
            return
        self._unplace(getattr(p, "place_key", None))

    def decode(self, items: list) -> list:
        groups: dict = {}
        for i, it in enumerate(items):
            groups.setdefault(it[0].device, []).append(i)
        out: list = [None] * len(items)

        def run(d, idx):
            for i, w in zip(idx, self.parts[d].decode([items[i] for i in idx])):
                out[i] = w

        self._each(groups, run)
        return out

    def _each(self, groups: dict, fn) -> None:
        """Run ``fn(device, indices)`` for every device group, concurrently when there are several (the C ABI releases
        the interpreter lock during its calls); the first failure is raised after all have finished."""
        errors = []

        def wrap(d, idx):
            try:
                fn(d, idx)
            except Exception as e:  # a failed device fails the call; the others still finish their part
                errors.append(e)

        if len(groups) == 1:
            (d, idx), = groups.items()
            wrap(d, idx)
        else:
            ts = [threading.Thread(target=wrap, args=(d, idx)) for d, idx in groups.items()]
            for t in ts:
                t.start()
            for t in ts:
                t.join()
        if errors:
            raise errors[0]
