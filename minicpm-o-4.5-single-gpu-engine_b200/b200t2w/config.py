"""The one place the Token2Wav DiT/CFM hyper-parameters live.

The reference reads these off the loaded ``stepaudio2`` estimator module (``engine/runtime/dit_fast.py:109-114,129``;
``engine/runtime/dit_graph.py:56-60``): depth = ``len(est.blocks)``, heads / head_dim from ``blocks[0].attn``, hidden =
``in_proj.out_features``, mel = ``in_proj.in_features // 4``, ``cfm.inference_cfg_rate``.  The checkpoint's
``assets/token2wav`` config that fixes their values is not available here, so the defaults below are the
reference-config values as published for Step-Audio2 / CosyVoice2 ``flow.yaml`` and are UNVERIFIED against the
checkpoint.  The oracle, the weight packer and the CUDA kernels all read them from a ``DiTConfig``; a correction is a
one-line change here.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, replace


@dataclass(frozen=True)
class DiTConfig:
    mel: int = 80                 # mel channels; in_proj takes [x, mu, spk, cond] = 4 * mel (dit_graph.py:59)
    hidden: int = 512             # in_proj.out_features (unverified)
    depth: int = 16               # len(est.blocks) (unverified; consistent with token2wav_batch.py:706's 18 GB figure)
    heads: int = 8                # blocks[i].attn.num_heads (unverified)
    head_dim: int = 64            # blocks[i].attn.head_dim (the reference's fused q/k norm requires 64, dit_kernels.py:139)
    mlp_ratio: float = 4.0        # DiTBlock MLP hidden = mlp_ratio * hidden (unverified)
    steps: int = 10               # Euler steps (Token2Wav n_timesteps, models/token2wav.py:250)
    cfg_rate: float = 0.7         # cfm.inference_cfg_rate (unverified)
    freq_dim: int = 256           # TimestepEmbedder sinusoid size (unverified)
    t_scale: float = 1000.0       # TimestepEmbedder multiplies t by this before the sinusoid (unverified)
    max_period: float = 10000.0   # sinusoid max period (unverified)
    eps_block: float = 1e-6       # norm1/norm2/norm3 (no affine) (unverified)
    eps_final: float = 1e-6       # final_layer.norm_final (no affine) (unverified)
    eps_qk: float = 1e-5          # attn.q_norm / attn.k_norm (affine, shared eps: dit_fast.py:134) (unverified)
    eps_conv: float = 1e-5        # conv.block[3] LayerNorm (affine) (unverified)
    conv_kernel: int = 3          # CausalConv1d kernel; 2 cached frames (token2wav_batch.py:82-97)

    @property
    def ffn(self) -> int:
        return int(self.hidden * self.mlp_ratio)

    @property
    def in_dim(self) -> int:
        return 4 * self.mel

    @property
    def conv_pad(self) -> int:
        return self.conv_kernel - 1

    @property
    def sm_scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)  # SDPA default scale (dit_fast.py:365 plans no sm_scale)

    def to_dict(self) -> dict:
        return asdict(self)

    def validate_for_kernels(self) -> None:
        """Shape limits of the sm_100a kernels (the oracle has none)."""
        if self.head_dim != 64:
            raise ValueError("the attention and q/k-norm kernels take head_dim == 64")
        if self.hidden != self.heads * self.head_dim:
            raise ValueError("hidden must equal heads * head_dim")
        if self.hidden % 128 or self.ffn % 128:
            raise ValueError("hidden and the MLP width must be multiples of 128")
        if self.hidden > 1024:
            raise ValueError("the row kernels hold one hidden row per warp (hidden <= 1024)")
        if self.mel > 128 or self.mel % 16:
            raise ValueError("mel must be a multiple of 16 and at most 128")
        if self.conv_kernel != 3:
            raise ValueError("the causal conv kernels take kernel size 3")


REFERENCE = DiTConfig()
"""The reference-config (unverified) used by every benchmark configuration."""

TINY = replace(REFERENCE, hidden=128, depth=2, heads=2, mlp_ratio=4.0)
"""A small config with the same kernel shapes class (head_dim 64), for fast golden fixtures and unit tests."""


def config_from_module(cfm, steps: int | None = None, base: DiTConfig = REFERENCE) -> DiTConfig:
    """The ``DiTConfig`` of a loaded ``CausalConditionalCFM``-like module, read off its attributes as the reference's
    ``FastDiT`` reads them (``engine/runtime/dit_fast.py:107-145``): depth = ``len(est.blocks)``; heads / head_dim from
    ``blocks[0].attn``; hidden = ``in_proj.out_features``; mel = ``in_proj.in_features // 4``; the MLP width from
    ``blocks[0].mlp.fc1``; the eps of ``norm1``, ``norm_final``, ``attn.q_norm`` and ``conv.block[3]``; the conv
    kernel from ``conv.block[1]``; the sinusoid size from ``t_embedder.mlp[0]``; ``cfm.inference_cfg_rate``.  The
    sinusoid's ``t_scale`` and ``max_period`` are not module attributes and come from ``base``.  Raises ValueError
    when the module contradicts itself (q_norm / k_norm eps, norm1 / norm2 / norm3 eps, mel vs ``out_channels``)."""
    est = cfm.estimator
    b0 = est.blocks[0]
    a = b0.attn
    hidden = int(est.in_proj.out_features)
    mel = int(est.in_proj.in_features) // 4
    if int(est.in_proj.in_features) != 4 * mel:
        raise ValueError("in_proj.in_features must be 4 * mel ([x, mu, spk, cond])")
    if int(getattr(est, "out_channels", mel)) != mel:
        raise ValueError("estimator.out_channels must equal in_proj.in_features // 4")
    if a.q_norm.eps != a.k_norm.eps:
        raise ValueError("attn.q_norm and attn.k_norm must share one eps")
    if not (b0.norm1.eps == b0.norm2.eps == b0.norm3.eps):
        raise ValueError("norm1 / norm2 / norm3 must share one eps")
    ffn = int(b0.mlp.fc1.out_features)
    return replace(
        base, mel=mel, hidden=hidden, depth=len(est.blocks), heads=int(a.num_heads), head_dim=int(a.head_dim),
        mlp_ratio=ffn / hidden, steps=int(steps) if steps is not None else base.steps,
        cfg_rate=float(cfm.inference_cfg_rate), freq_dim=int(est.t_embedder.mlp[0].in_features),
        eps_block=float(b0.norm1.eps), eps_final=float(est.final_layer.norm_final.eps), eps_qk=float(a.q_norm.eps),
        eps_conv=float(b0.conv.block[3].eps), conv_kernel=int(b0.conv.block[1].kernel_size[0]))


def t_schedule(steps: int):
    """The solver's t recurrence in fp32, as ``BatchedToken2Wav._solve`` runs it (token2wav_batch.py:669-693):
    ``t_span = 1 - cos(linspace(0, 1, S + 1) * pi / 2)``; ``t`` starts at ``t_span[0]`` and is accumulated as ``t + dt``
    (not read from ``t_span``), ``dt = t_span[step + 1] - t``.  Returns (ts, dts) as python floats of the fp32 values."""
    import torch

    t_span = torch.linspace(0, 1, steps + 1, dtype=torch.float32)
    t_span = 1 - torch.cos(t_span * 0.5 * torch.pi)
    t, dt = t_span[0].clone(), t_span[1] - t_span[0]
    ts, dts = [], []
    for step in range(1, steps + 1):
        ts.append(float(t))
        dts.append(float(dt))
        t = t + dt
        if step < steps:
            dt = t_span[step + 1] - t
    return ts, dts


@dataclass(frozen=True)
class EncoderConfig:
    """The flow encoder's hyper-parameters (``UpsampleConformerEncoderV2`` of ``stepaudio2``; the reference reads them
    off the module: ``len(enc.encoders)``, ``len(enc.up_encoders)``, ``enc.up_layer.stride``,
    ``enc.pre_lookahead_layer.pre_lookahead_len``, the attention cache's heads and ``2 * d_k``,
    ``engine/runtime/token2wav_batch.py:408-418``).  The values are the published CosyVoice2 / Step-Audio2 ``flow.yaml``
    encoder (512 wide, 8 heads, 2048-wide swish feed-forward, 6 + 4 conformer blocks without conv module or macaron,
    ESPnet relative positions, linear input layer, pre-norm) and are UNVERIFIED against the checkpoint."""
    vocab: int = 6561             # flow.input_embedding rows (speech tokens, unverified)
    hidden: int = 512             # encoder output_size and input_size (unverified)
    heads: int = 8                # attention heads (unverified)
    head_dim: int = 64            # d_k; the attention cache holds [k | v] = 2 d_k per frame
    ffn: int = 2048               # linear_units (unverified)
    blocks1: int = 6              # len(enc.encoders) (unverified)
    blocks2: int = 4              # len(enc.up_encoders) (unverified)
    stride: int = 2               # enc.up_layer.stride: two mel frames per token
    lookahead: int = 3            # enc.pre_lookahead_layer.pre_lookahead_len (engine/token2wav_chunker.py:20)
    mel: int = 80                 # encoder_proj output (the DiT's mu channels)
    spk_dim: int = 192            # spk_embed_affine_layer input (CAMPPlus embedding, unverified)
    eps_layer: float = 1e-12      # norm_mha / norm_ff of each conformer layer (unverified)
    eps_embed: float = 1e-5       # embed / up_embed LayerNorm (unverified)
    eps_after: float = 1e-5       # after_norm (unverified)
    leaky_slope: float = 0.01     # pre-lookahead conv1 activation (F.leaky_relu default)
    max_period: float = 10000.0   # relative positional encoding sinusoid base

    @property
    def conv1_kernel(self) -> int:
        return self.lookahead + 1

    @property
    def up_kernel(self) -> int:
        return 2 * self.stride + 1

    @property
    def cnn_cache(self) -> int:
        """Frames of the conv cache: 2 of the pre-lookahead conv2, 2 * stride of the upsampling conv."""
        return 2 + 2 * self.stride

    def validate_for_kernels(self) -> None:
        if self.head_dim != 64 or self.hidden != self.heads * self.head_dim:
            raise ValueError("the attention kernel takes head_dim == 64 and hidden == heads * 64")
        if self.hidden % 128 or self.ffn % 128 or self.hidden > 1024:
            raise ValueError("hidden and ffn must be multiples of 128, hidden <= 1024")
        if self.mel != 80:
            raise ValueError("encoder_proj runs on the 80-column GEMM tile")
        if self.stride != 2 or self.lookahead != 3:
            raise ValueError("the conv kernels take stride 2 and a 3-frame lookahead")


ENCODER = EncoderConfig()
"""The reference-config (unverified) flow encoder."""

ENCODER_TINY = replace(ENCODER, hidden=128, heads=2, ffn=256, blocks1=2, blocks2=2, spk_dim=32)
"""A small encoder with the same kernel shape class, for fast golden fixtures."""


@dataclass(frozen=True)
class HiFTConfig:
    """The HiFT vocoder's hyper-parameters (``stepaudio2``'s ``HiFTGenerator``; the reference reads ``num_upsamples``,
    ``num_kernels``, ``istft_params``, ``lrelu_slope``, ``audio_limit``, ``f0_upsamp.scale_factor`` and the source's
    ``l_sin_gen`` fields off the module, ``engine/models/token2wav.py:112-245``).  The values are the published
    CosyVoice2 ``hift.yaml`` (24 kHz, 512 base channels, upsampling 8 x 5 x 3 with an n_fft 16 / hop 4 iSTFT, 8
    harmonics) and are UNVERIFIED against the checkpoint."""
    mel: int = 80
    channels: int = 512                      # base_channels (unverified)
    upsample_rates: tuple = (8, 5, 3)
    upsample_kernels: tuple = (16, 11, 7)
    resblock_kernels: tuple = (3, 7, 11)
    source_kernels: tuple = (7, 7, 11)       # source_resblock_kernel_sizes (unverified)
    dilations: tuple = (1, 3, 5)             # every ResBlock's dilations
    n_fft: int = 16
    hop: int = 4
    harmonics: int = 8                       # nb_harmonics
    sample_rate: int = 24000
    nsf_alpha: float = 0.1                   # sine amplitude
    nsf_sigma: float = 0.003                 # additive noise std of voiced samples
    voiced_threshold: float = 10.0
    lrelu_slope: float = 0.1
    audio_limit: float = 0.99
    f0_channels: int = 512                   # ConvRNNF0Predictor cond_channels (unverified)
    f0_layers: int = 5

    @property
    def upsample_scale(self) -> int:
        """Waveform samples per mel frame: the product of the upsampling rates times the iSTFT hop (480)."""
        return int(math.prod(self.upsample_rates)) * self.hop


HIFT = HiFTConfig()
"""The reference-config (unverified) vocoder."""

HIFT_TINY = replace(HIFT, channels=256, f0_channels=128, f0_layers=2)
"""A narrower vocoder with the same stage structure (stages of 128, 64 and 32 channels), for fast golden fixtures."""
