"""CPU fp32 oracle of the Token2Wav HiFT vocoder (mel -> 24 kHz waveform).  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this module, and only as
the checker: the product (the ``b200t2w`` package and its CUDA library) never calls into it.

1. A restatement of the third-party vocoder the reference engine drives (``stepaudio2``'s ``HiFTGenerator`` with
   ``SourceModuleHnNSF2`` / ``SineGen2`` and the ``ConvRNNF0Predictor``, from ``minicpmo-utils==1.0.6``, absent here:
   ``engine/env/engine.lock:46``).  The module carries the attribute names and call forms the engine reads
   (``engine/models/token2wav.py:112-245``): ``f0_predictor(mel)``, ``f0_upsamp`` (its ``scale_factor``), ``m_source``
   (``l_sin_gen`` with ``harmonic_num``, ``dim``, ``sampling_rate``, ``upsample_scale``, ``sine_amp``, ``noise_std``,
   ``flag_for_pulse``, ``_f02uv``; ``l_linear``, ``l_tanh``), ``_stft``, ``conv_pre``, ``num_upsamples``,
   ``lrelu_slope``, ``ups``, ``reflection_pad``, ``source_downs``, ``source_resblocks``, ``num_kernels``,
   ``resblocks``, ``conv_post``, ``istft_params``, ``stft_window``, ``audio_limit``.  The arithmetic follows the
   published CosyVoice2 / HiFi-GAN NSF algorithms: a 5-layer conv + ELU f0 predictor with a linear head and |.|; three
   transposed-conv upsampling stages (rates 8, 5, 3, kernels 16, 11, 7) each adding a strided-conv + ResBlock branch of
   the source's STFT, then the average of three ResBlocks (kernels 3, 7, 11, dilations 1, 3, 5; Snake activations
   x + sin^2(a x) / a); a reflection pad, conv_post, exp / sin of its two halves and an inverse STFT (n_fft 16, hop 4,
   Hann).  Weight normalisation is folded into plain weights (the reference's lean form evaluates it once).  Its
   fidelity to the real package is unpinned (the package is absent).
2. ``hift_forward_noise`` / ``hift_decode`` / ``istft`` restate the reference's own driver functions
   (``engine/models/token2wav.py:112-245``) per stream, and ``vocode_window`` restates ``BatchedToken2Wav._vocode``'s
   per-stream bookkeeping (``engine/runtime/token2wav_batch.py:813-848``: the 8-frame mel cache, the 3840-sample source
   and speech caches, the Hamming cross-fade, the held-back tail and the leading silence of a first window); pinned by
   ``tests/golden/make_hift_golden.py``, which runs the reference's own functions on this module.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

_HERE = os.path.dirname(os.path.abspath(__file__))
_PKG = os.path.join(os.path.dirname(_HERE), "minicpm-o-4.5-single-gpu-engine_b200")
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

from b200t2w.config import HiFTConfig  # noqa: E402

MEL_CACHE = 8        # engine/models/token2wav.py:35
SOURCE_CACHE = MEL_CACHE * 480


class Snake(nn.Module):
    """x + 1 / (alpha + 1e-9) * sin(alpha x)^2, one alpha per channel ([B, C, T] input)."""

    def __init__(self, channels: int):
        super().__init__()
        self.alpha = nn.Parameter(torch.ones(channels))

    def forward(self, x):
        a = self.alpha[None, :, None]
        return x + 1.0 / (a + 1e-9) * torch.pow(torch.sin(x * a), 2)


def _pad(k: int, d: int) -> int:
    return (k * d - d) // 2


class ResBlock(nn.Module):
    """HiFi-GAN residual block: per dilation d, x += conv2(snake2(conv1_d(snake1(x)))) ("same" padding)."""

    def __init__(self, channels: int, k: int, dilations):
        super().__init__()
        self.convs1 = nn.ModuleList([nn.Conv1d(channels, channels, k, 1, dilation=d, padding=_pad(k, d)) for d in dilations])
        self.convs2 = nn.ModuleList([nn.Conv1d(channels, channels, k, 1, dilation=1, padding=_pad(k, 1)) for _ in dilations])
        self.activations1 = nn.ModuleList([Snake(channels) for _ in dilations])
        self.activations2 = nn.ModuleList([Snake(channels) for _ in dilations])

    def forward(self, x):
        for c1, c2, a1, a2 in zip(self.convs1, self.convs2, self.activations1, self.activations2):
            x = c2(a2(c1(a1(x)))) + x
        return x


class ConvRNNF0Predictor(nn.Module):
    def __init__(self, cfg: HiFTConfig):
        super().__init__()
        layers = []
        for i in range(cfg.f0_layers):
            layers += [nn.Conv1d(cfg.mel if i == 0 else cfg.f0_channels, cfg.f0_channels, 3, 1, 1), nn.ELU()]
        self.condnet = nn.Sequential(*layers)
        self.classifier = nn.Linear(cfg.f0_channels, 1)

    def forward(self, x):
        x = self.condnet(x).transpose(1, 2)
        return torch.abs(self.classifier(x).squeeze(-1))


class SineGen2(nn.Module):
    """The harmonic sine source's parameters (the reference reimplements its forward with given noise)."""

    def __init__(self, cfg: HiFTConfig):
        super().__init__()
        self.sine_amp, self.noise_std, self.harmonic_num = cfg.nsf_alpha, cfg.nsf_sigma, cfg.harmonics
        self.dim = cfg.harmonics + 1
        self.sampling_rate, self.voiced_threshold = cfg.sample_rate, cfg.voiced_threshold
        self.flag_for_pulse = False
        self.upsample_scale = cfg.upsample_scale

    def _f02uv(self, f0):
        return (f0 > self.voiced_threshold).type(torch.float32)


class SourceModuleHnNSF2(nn.Module):
    def __init__(self, cfg: HiFTConfig):
        super().__init__()
        self.sine_amp, self.noise_std = cfg.nsf_alpha, cfg.nsf_sigma
        self.l_sin_gen = SineGen2(cfg)
        self.l_linear = nn.Linear(cfg.harmonics + 1, 1)
        self.l_tanh = nn.Tanh()


class HiFTGenerator(nn.Module):
    def __init__(self, cfg: HiFTConfig):
        super().__init__()
        self.cfg = cfg
        self.istft_params = {"n_fft": cfg.n_fft, "hop_len": cfg.hop}
        self.lrelu_slope, self.audio_limit = cfg.lrelu_slope, cfg.audio_limit
        self.num_kernels = len(cfg.resblock_kernels)
        self.num_upsamples = len(cfg.upsample_rates)
        self.m_source = SourceModuleHnNSF2(cfg)
        self.f0_upsamp = nn.Upsample(scale_factor=float(cfg.upsample_scale))
        C = cfg.channels
        self.conv_pre = nn.Conv1d(cfg.mel, C, 7, 1, padding=3)
        self.ups = nn.ModuleList([nn.ConvTranspose1d(C // 2 ** i, C // 2 ** (i + 1), k, u, padding=(k - u) // 2)
                                  for i, (u, k) in enumerate(zip(cfg.upsample_rates, cfg.upsample_kernels))])
        self.source_downs, self.source_resblocks = nn.ModuleList(), nn.ModuleList()
        cum = np.cumprod([1] + list(cfg.upsample_rates[::-1][:-1]))[::-1]  # 15, 3, 1 for rates 8, 5, 3
        for i, (u, k) in enumerate(zip(cum, cfg.source_kernels)):
            ch = C // 2 ** (i + 1)
            u = int(u)
            self.source_downs.append(nn.Conv1d(cfg.n_fft + 2, ch, 1, 1) if u == 1 else
                                     nn.Conv1d(cfg.n_fft + 2, ch, u * 2, u, padding=u // 2))
            self.source_resblocks.append(ResBlock(ch, k, cfg.dilations))
        self.resblocks = nn.ModuleList([ResBlock(C // 2 ** (i + 1), k, cfg.dilations)
                                        for i in range(self.num_upsamples) for k in cfg.resblock_kernels])
        self.conv_post = nn.Conv1d(C // 2 ** self.num_upsamples, cfg.n_fft + 2, 7, 1, padding=3)
        self.reflection_pad = nn.ReflectionPad1d((1, 0))
        self.register_buffer("stft_window", torch.hann_window(cfg.n_fft, periodic=True), persistent=False)
        self.f0_predictor = ConvRNNF0Predictor(cfg)

    def _stft(self, x):
        spec = torch.stft(x, self.cfg.n_fft, self.cfg.hop, self.cfg.n_fft, window=self.stft_window.to(x.device),
                          return_complex=True)
        spec = torch.view_as_real(spec)
        return spec[..., 0], spec[..., 1]


def build_hift(cfg: HiFTConfig, seed: int = 0) -> HiFTGenerator:
    """Random-init vocoder: ``torch.manual_seed(seed)``, PyTorch's default init in construction order, then every Snake
    alpha exp(0.3 N(0, 1)) (positive, not all ones), conv_post's weight scaled by 0.3 (its exp half stays below the
    100 clip and the waveform below the 0.99 clamp for most samples) and the f0 head's bias set so that roughly half the
    frames are voiced (f0 > 10 Hz: both branches of the source are exercised)."""
    torch.manual_seed(seed)
    m = HiFTGenerator(cfg)
    with torch.no_grad():
        for mod in m.modules():
            if isinstance(mod, Snake):
                mod.alpha.copy_(torch.exp(0.3 * torch.randn_like(mod.alpha)))
        m.conv_post.weight.mul_(0.3)
        # the f0 head: scaled so f0 spans tens of Hz, shifted so the median frame sits at the voiced threshold
        head = m.f0_predictor.classifier
        head.weight.mul_(40.0)
        probe = torch.randn(4, cfg.mel, 64, generator=torch.Generator().manual_seed(123)) - 2.0
        raw = head(m.f0_predictor.condnet(probe).transpose(1, 2)).flatten()
        head.bias.add_(cfg.voiced_threshold - raw.median())
    return m.eval()


# ---- the reference's driver functions, per stream (engine/models/token2wav.py:112-245)


def hift_samples(hift, mel_frames: int) -> int:
    return int(mel_frames * hift.f0_upsamp.scale_factor)


def hift_noise(hift, seed: int, n_samples: int):
    """``hift_noise`` for one row: the initial phases ``rand`` then the additive noise ``randn`` drawn channel-major."""
    gen = hift.m_source.l_sin_gen
    g = torch.Generator().manual_seed(int(seed))
    rand_ini = torch.rand(1, gen.dim, generator=g)
    noise = torch.randn(1, gen.dim, n_samples, generator=g).transpose(1, 2)
    return rand_ini, noise


def istft(spec, n_fft: int, hop: int, window):
    frames = torch.fft.irfft(spec, n=n_fft, dim=1) * window[None, :, None]
    T = frames.shape[2]
    total = (T - 1) * hop + n_fft
    y = F.fold(frames, output_size=(1, total), kernel_size=(1, n_fft), stride=(1, hop))[:, 0, 0]
    env = F.fold((window ** 2)[None, :, None].expand(1, n_fft, T), output_size=(1, total), kernel_size=(1, n_fft),
                 stride=(1, hop))[0, 0, 0]
    half = n_fft // 2
    return (y / env)[:, half:total - half]


def hift_decode(hift, x, s):
    s_re, s_im = hift._stft(s.squeeze(1))
    s_stft = torch.cat([s_re, s_im], dim=1)
    x = hift.conv_pre(x)
    for i in range(hift.num_upsamples):
        x = F.leaky_relu(x, hift.lrelu_slope)
        x = hift.ups[i](x)
        if i == hift.num_upsamples - 1:
            x = hift.reflection_pad(x)
        x = x + hift.source_resblocks[i](hift.source_downs[i](s_stft))
        xs = None
        for j in range(hift.num_kernels):
            r = hift.resblocks[i * hift.num_kernels + j](x)
            xs = r if xs is None else xs + r
        x = xs / hift.num_kernels
    x = F.leaky_relu(x)
    x = hift.conv_post(x)
    nf = hift.istft_params["n_fft"]
    magnitude = torch.clip(torch.exp(x[:, :nf // 2 + 1, :]), max=1e2)
    phase = torch.sin(x[:, nf // 2 + 1:, :])
    y = istft(torch.complex(magnitude * torch.cos(phase), magnitude * torch.sin(phase)), nf, hift.istft_params["hop_len"],
              hift.stft_window)
    return torch.clamp(y, -hift.audio_limit, hift.audio_limit)


@torch.no_grad()
def hift_forward_noise(hift, mel, cache_source, rand_ini, noise):
    """mel [B, 80, F], cache_source [B, 1, n] (n = 0 or SOURCE_CACHE) -> (speech [B, F * 480], source [B, 1, F * 480])."""
    f0 = hift.f0_predictor(mel)
    s = hift.f0_upsamp(f0[:, None]).transpose(1, 2)
    src = hift.m_source
    gen = src.l_sin_gen
    fn = torch.multiply(s, torch.arange(1, gen.harmonic_num + 2, dtype=torch.float32)[None, None, :])
    rad = (fn / gen.sampling_rate) % 1
    rand_ini = rand_ini.clone()
    rand_ini[:, 0] = 0
    rad[:, 0, :] = rad[:, 0, :] + rand_ini
    rad = F.interpolate(rad.transpose(1, 2), scale_factor=1 / gen.upsample_scale, mode="linear").transpose(1, 2)
    phase = torch.cumsum(rad, dim=1) * 2 * np.pi
    phase = F.interpolate(phase.transpose(1, 2) * gen.upsample_scale, scale_factor=gen.upsample_scale,
                          mode="linear").transpose(1, 2)
    sine = torch.sin(phase) * gen.sine_amp
    uv = gen._f02uv(fn[..., :1])
    sine = sine * uv + (uv * gen.noise_std + (1 - uv) * gen.sine_amp / 3) * noise
    s = src.l_tanh(src.l_linear(sine)).transpose(1, 2)
    if cache_source.shape[2] != 0:
        s[:, :, :cache_source.shape[2]] = cache_source
    return hift_decode(hift, mel, s), s


def fade_in_out(fade_in, fade_out, window):
    n = int(window.shape[0] / 2)
    out = fade_in.clone()
    out[..., :n] = fade_in[..., :n] * window[:n] + fade_out[..., -n:] * window[n:]
    return out


class HiftStream:
    """One stream's vocoder caches: the last 8 mel frames, 3840 source samples and 3840 speech samples."""

    def __init__(self, mel_dim: int = 80):
        self.mel = torch.zeros(1, mel_dim, 0)
        self.source = torch.zeros(1, 1, 0)
        self.speech = torch.zeros(1, 0)
        self.chunks = 0


@torch.no_grad()
def vocode_window(hift, st: HiftStream, mel, seed: int, last: bool, noise_fn=None):
    """One window's mel [80, T] -> its samples, as ``BatchedToken2Wav._vocode`` handles one stream: the mel after the
    cached frames, HiFT with the row's seeded noise, the cross-fade with the cached speech, the caches updated, and the
    last 3840 samples held back (a first window shifted by 3840 samples of silence) unless the window is final.
    ``noise_fn(seed, n_samples) -> (rand_ini [1, dim], noise [1, n, dim])`` draws the noise in place of the CPU
    generator (the reference draws on the vocoder's device)."""
    M = torch.cat([st.mel, mel[None]], dim=2)
    rand_ini, noise = (noise_fn or (lambda s, n: hift_noise(hift, s, n)))(seed, hift_samples(hift, M.shape[2]))
    speech, source = hift_forward_noise(hift, M, st.source, rand_ini, noise)
    first = st.source.shape[2] == 0
    window = torch.from_numpy(np.hamming(2 * SOURCE_CACHE))  # float64, as the reference keeps it
    if not first:
        speech = fade_in_out(speech, st.speech, window)
    st.mel, st.source, st.speech = M[..., -MEL_CACHE:].clone(), source[:, :, -SOURCE_CACHE:].clone(), \
        speech[:, -SOURCE_CACHE:].clone()
    st.chunks += 1
    sp = speech[0]
    if not last:
        sp = torch.cat([torch.zeros(SOURCE_CACHE), sp[:-SOURCE_CACHE]]) if first else sp[:-SOURCE_CACHE]
    return sp


def chunk_noise_seed(noise_seed: int, chunk: int) -> int:
    """engine/models/token2wav.py:108-109."""
    return (noise_seed * 1_000_003 + chunk) & ((1 << 63) - 1)


def state_dict_np(m) -> dict:
    return {k: v.detach().float().numpy() for k, v in m.state_dict().items()}

