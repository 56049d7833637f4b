"""Host side of the B200 HiFT vocoder (mel -> 24 kHz waveform), through the C ABI of ``libt2w_b200.so``.

The reference vocodes a decode call's windows in ``BatchedToken2Wav._vocode`` (``engine/runtime/token2wav_batch.py:
813-848``) with ``hift_forward`` (``engine/models/token2wav.py:230-245``) and keeps each stream's ``hift_cache`` (mel /
source / speech tails).  ``B200HiFT`` keeps those caches in the library: a stream is a handle; ``vocode(handles, mels,
lasts)`` runs every window of the call in one library call and returns each window's samples exactly as ``_vocode``
returns them (held-back tail, leading silence of a first window, the Hamming cross-fade).  The source noise of a
stream's chunk is drawn here as the reference draws it (``hift_noise``: a generator seeded with the chunk's seed, the
initial phases then the additive noise, on the vocoder's device).  All arithmetic runs in the CUDA library; a missing
library or a non-sm_100 device raises.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import lib as L
from .config import HIFT, HiFTConfig


def chunk_noise_seed(noise_seed: int, chunk: int) -> int:
    """A stream's chunk seed (engine/models/token2wav.py:108-109)."""
    return (noise_seed * 1_000_003 + chunk) & ((1 << 63) - 1)


PARTS = ("ups", "src", "res")  # a stage's transposed convolution, its source branch, its ResBlocks


def tf32_parts(spec, stages: int = 3) -> int:
    """The ``t2w_hift_config.tf32_parts`` mask (bit 3 s + p) of a ``decode_tf32`` value as the reference reads it
    (``tf32_stages``, engine/models/token2wav.py:145-158): True for every part of every stage, False / None / empty for
    none, else a list of stage indices (all parts of that stage) and ``"<stage>:<part>"`` entries, part one of
    ``ups``, ``src``, ``res``."""
    if spec is True:
        return (1 << (3 * stages)) - 1
    if not spec:
        return 0
    mask = 0
    for e in spec:
        i, _, part = str(e).partition(":")
        if not 0 <= int(i) < stages or part not in ("",) + PARTS:
            raise ValueError(f"tf32 entry {e!r}: a stage index < {stages} or '<stage>:<part>' with a part of {PARTS}")
        for q in ((PARTS.index(part),) if part else range(3)):
            mask |= 1 << (3 * int(i) + q)
    return mask


def hift_weight_names(cfg: HiFTConfig) -> list:
    """State-dict paths of a HiFTGenerator in the order ``t2w_hift_create`` takes them (include/t2w_b200.h)."""
    n = []
    for l in range(cfg.f0_layers):
        n += [f"f0_predictor.condnet.{2 * l}.weight", f"f0_predictor.condnet.{2 * l}.bias"]
    n += ["f0_predictor.classifier.weight", "f0_predictor.classifier.bias", "m_source.l_linear.weight",
          "m_source.l_linear.bias", "conv_pre.weight", "conv_pre.bias"]
    for s in range(3):
        n += [f"ups.{s}.weight", f"ups.{s}.bias"]

    def block(p):
        out = []
        for d in range(3):
            out += [f"{p}.convs1.{d}.weight", f"{p}.convs1.{d}.bias"]
        for d in range(3):
            out += [f"{p}.convs2.{d}.weight", f"{p}.convs2.{d}.bias"]
        out += [f"{p}.activations1.{d}.alpha" for d in range(3)]
        out += [f"{p}.activations2.{d}.alpha" for d in range(3)]
        return out

    for s in range(3):
        n += [f"source_downs.{s}.weight", f"source_downs.{s}.bias"] + block(f"source_resblocks.{s}")
    for b in range(9):
        n += block(f"resblocks.{b}")
    n += ["conv_post.weight", "conv_post.bias"]
    return n


class B200HiFT:
    """The HiFT vocoder on one sm_100 GPU.  ``weights``: fp32 state dict of a HiFTGenerator (weight normalisation
    folded); ``max_frames``: a window's mel frames at most, with the 8 cached ones (<= 512).  ``tf32``: the upsampling
    stages on TF32 tensor cores, the reference's ``decode_tf32`` option and values (True, or a list of stages and
    ``"<stage>:<part>"`` entries, ``tf32_parts``); False keeps every convolution in strict fp32 (the reference's
    default) on CUDA cores.  ``split_fp32``: every convolution on the tensor cores in split form instead (operands as
    pairs of TF32 values, hi W_hi + hi W_lo + lo W_hi: fp32-level products, the reference's fp32 numerics at
    tensor-core speed); ``tf32`` is then ignored.  ``use_graphs``: each call replays a CUDA graph of its launches per
    call structure (the reference's ``t2w_graphs`` / ``HiFTGraphs``), captured the second time a structure is seen;
    calls then have to stay ordered on one stream."""

    def __init__(self, cfg: HiFTConfig, weights: dict, device="cuda", max_frames: int = 128, n_streams: int = 256,
                 tf32=True, split_fp32: bool = False, use_graphs: bool = False):
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("B200HiFT needs a CUDA device (no CPU fallback)")
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", idx)
        self.lib = L.load()
        if not self.lib.t2w_device_ok(idx):
            raise RuntimeError(f"cuda:{idx} is not an sm_100 GPU: the B200 kernels cannot run there")
        names = hift_weight_names(cfg)
        missing = [k for k in names if k not in weights]
        if missing:
            raise KeyError(f"HiFT weights lack {missing[:4]}")
        c = L.HiftConfig()
        c.mel, c.channels, c.f0_channels, c.f0_layers = cfg.mel, cfg.channels, cfg.f0_channels, cfg.f0_layers
        c.harmonics, c.sample_rate, c.n_fft, c.hop = cfg.harmonics, cfg.sample_rate, cfg.n_fft, cfg.hop
        for f, v in (("up_rates", cfg.upsample_rates), ("up_kernels", cfg.upsample_kernels),
                     ("res_kernels", cfg.resblock_kernels), ("source_kernels", cfg.source_kernels),
                     ("dilations", cfg.dilations)):
            setattr(c, f, (ctypes.c_int32 * 3)(*v))
        c.nsf_alpha, c.nsf_sigma, c.voiced_threshold = cfg.nsf_alpha, cfg.nsf_sigma, cfg.voiced_threshold
        c.lrelu_slope, c.audio_limit = cfg.lrelu_slope, cfg.audio_limit
        mask = 0 if split_fp32 else tf32_parts(tf32)
        c.tf32 = 2 if split_fp32 else (1 if mask else 0)
        c.tf32_parts = mask
        self.tf32 = bool(mask)
        self.tf32_parts = mask
        self.split_fp32 = bool(split_fp32)
        self.use_graphs = bool(use_graphs)
        with torch.cuda.device(self.device):
            w = [weights[k].detach().to(self.device, torch.float32).contiguous() for k in names]
            ptrs = (ctypes.c_void_p * len(w))(*[t.data_ptr() for t in w])
            h = ctypes.c_void_p()
            L.call("t2w_hift_create", ctypes.byref(c), ptrs, len(w), max_frames, n_streams, ctypes.byref(h))
        self.handle = h
        self.max_frames = max_frames
        self._seeds: dict = {}  # handle -> [noise seed, chunks so far]
        self._gens: dict = {}  # handle -> its device generator, re-seeded for every chunk
        self._side = None  # the stream the seeded noise is drawn on (created on first use)

    @classmethod
    def from_module(cls, hift, cfg: HiFTConfig = HIFT, **kw) -> "B200HiFT":
        return cls(cfg, {k: v.detach().float() for k, v in hift.state_dict().items()}, **kw)

    @classmethod
    def for_decode_tf32(cls, hift, decode_tf32=False, cfg: HiFTConfig = HIFT, **kw) -> "B200HiFT":
        """The vocoder for a reference config's ``t2w_hift_decode_tf32`` value (engine/runtime/t2w_worker.py:654,
        ``BatchedToken2Wav(hift_decode_tf32=...)``): False / None — the reference's strict fp32 — gives the split-form
        fp32 mode on the tensor cores; True or a list of stages / ``"<stage>:<part>"`` the same TF32 parts."""
        if not decode_tf32:
            return cls.from_module(hift, cfg, split_fp32=True, **kw)
        return cls.from_module(hift, cfg, tf32=decode_tf32, **kw)

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.t2w_hift_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self) -> None:
        L.check("t2w_hift_check", self.lib.t2w_hift_check(self.handle))

    @property
    def counts(self) -> dict:
        """Calls so far: graph replays, graph captures, eager calls."""
        v = [ctypes.c_int64() for _ in range(3)]
        L.call("t2w_hift_counts", self.handle, *[ctypes.byref(x) for x in v])
        return {"replays": v[0].value, "captures": v[1].value, "eager": v[2].value}

    def new_stream(self, noise_seed: int = 0) -> int:
        h = ctypes.c_int32()
        L.call("t2w_hift_stream_new", self.handle, ctypes.byref(h))
        self._seeds[h.value] = [int(noise_seed), 0]
        self._gens[h.value] = torch.Generator(device=self.device)
        return h.value

    def release(self, handle: int) -> None:
        L.call("t2w_hift_stream_release", self.handle, int(handle))
        self._seeds.pop(int(handle), None)
        self._gens.pop(int(handle), None)

    def _draw_stream(self) -> torch.cuda.Stream:
        if self._side is None:
            self._side = torch.cuda.Stream(device=self.device)
        return self._side

    def _draw(self, g: torch.Generator, seed: int, rand_ini: torch.Tensor, noise: torch.Tensor) -> None:
        """``hift_noise`` for one row, in place: ``rand_ini`` [1, dim] then ``noise`` [1, dim, n] drawn as a fresh
        generator seeded with ``seed`` draws them (``manual_seed`` restarts a CUDA generator's Philox offset at 0, and
        ``uniform_`` / ``normal_`` are what ``torch.rand`` / ``torch.randn`` fill with)."""
        g.manual_seed(int(seed))
        rand_ini.uniform_(0.0, 1.0, generator=g)
        noise.normal_(0.0, 1.0, generator=g)

    def vocode(self, handles, mels, lasts, noise=None, source=None) -> list:
        """One window per stream: ``mels[i]`` [mel, T_i], ``lasts[i]`` the final flag.  Returns each window's samples
        (device fp32 tensors, ``_vocode``'s output).  ``noise``: optional per-window (rand_ini [1, dim], noise [1, dim,
        480 F_i]) in place of the seeded draws (tests).  ``source``: optional device fp32 tensor of sum 480 F_i floats
        that receives the windows' harmonic source signals, back to back."""
        if len(mels) != len(handles) or len(lasts) != len(handles):
            raise ValueError("one mel and one final flag per stream")
        Ts = [int(m.shape[1]) for m in mels]
        packed = torch.cat([m.t() for m in mels]).to(self.device, torch.float32).contiguous()
        return self.vocode_packed(handles, packed, Ts, lasts, noise, source=source)

    def vocode_packed(self, handles, mel_rows: torch.Tensor, Ts, lasts, noise=None, flat: bool = False, source=None):
        """``vocode`` on the windows' mel rows token-major ``[sum T_i, mel]`` (the solve's output layout).  ``flat``:
        return ``(samples, counts)``, every window's samples back to back in one device tensor, instead of the list."""
        n = len(handles)
        hs = L.i32_array(handles)
        ts = L.i32_array(Ts)
        ls = (ctypes.c_uint8 * n)(*[1 if x else 0 for x in lasts])
        per = (ctypes.c_int64 * n)()
        frames = (ctypes.c_int32 * n)()
        tot = self.lib.t2w_vocode_samples(self.handle, n, hs, ts, ls, per, frames)
        if tot < 0:
            raise L.T2WError("t2w_vocode_samples", -1)
        dim = self.cfg.harmonics + 1
        ready = None
        with torch.cuda.device(self.device):
            if noise is None:
                # every row's draws straight into the packed buffers the library reads, on a stream of their own: the
                # call waits for them only before its harmonic source, so they overlap its first kernels
                main = torch.cuda.current_stream()
                side = main if torch.cuda.is_current_stream_capturing() else self._draw_stream()
                samples = [480 * frames[i] for i in range(n)]
                with torch.cuda.stream(side):
                    rand_ini = torch.empty(n, dim, dtype=torch.float32, device=self.device)
                    nz = torch.empty(dim * sum(samples), dtype=torch.float32, device=self.device)
                    o = 0
                    for i, h in enumerate(handles):
                        seed, chunks = self._seeds[int(h)]
                        self._draw(self._gens[int(h)], chunk_noise_seed(seed, chunks), rand_ini[i:i + 1],
                                   nz[o:o + dim * samples[i]].view(1, dim, samples[i]))
                        o += dim * samples[i]
                if side is not main:
                    ready = torch.cuda.Event()
                    ready.record(side)
                    rand_ini.record_stream(main)  # the buffers live until the vocoder's stream has read them
                    nz.record_stream(main)
            else:
                rand_ini = torch.cat([d[0].reshape(1, dim) for d in noise]).to(self.device, torch.float32).contiguous()
                nz = torch.cat([d[1].reshape(-1) for d in noise]).to(self.device, torch.float32).contiguous()
            out = torch.empty(int(tot), dtype=torch.float32, device=self.device)
            if source is not None and (source.dtype != torch.float32 or source.device != self.device or
                                       source.numel() < 480 * sum(frames[i] for i in range(n)) or
                                       not source.is_contiguous()):
                raise ValueError("source: a contiguous fp32 tensor on the vocoder's device of sum 480 F_i floats")
            src = ctypes.c_void_p(source.data_ptr()) if source is not None else None
            b = L.VocodeBatch(n, hs, ts, ls, ctypes.c_void_p(mel_rows.data_ptr()), ctypes.c_void_p(rand_ini.data_ptr()),
                              ctypes.c_void_p(nz.data_ptr()), ctypes.c_void_p(out.data_ptr()), src, None,
                              1 if self.use_graphs else 0,
                              ctypes.c_void_p(ready.cuda_event) if ready is not None else None)
            L.call("t2w_vocode", self.handle, ctypes.byref(b), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        for h in handles:
            self._seeds[int(h)][1] += 1
        if flat:
            return out, list(per)
        res, o = [], 0
        for i in range(n):
            res.append(out[o:o + per[i]])
            o += per[i]
        return res

    def vocode_numpy(self, handles, mels, lasts) -> list:
        """``vocode`` with one device-to-host copy for the call (the reference's ``_vocode`` returns numpy arrays)."""
        outs = self.vocode(handles, mels, lasts)
        flat = torch.cat(outs).cpu().numpy() if outs else np.zeros(0, np.float32)
        res, o = [], 0
        for x in outs:
            res.append(flat[o:o + x.numel()])
            o += x.numel()
        return res
