"""CPU fp32 oracle of the Token2Wav DiT/CFM flow-matching solve.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may import this module,
and only as the checker or the timed CPU baseline: the product (the ``b200t2w`` package and its CUDA library) never
calls into it.

Two halves:

1. A restatement of the third-party estimator modules the reference engine drives (``stepaudio2.cosyvoice2.flow.
   decoder_dit`` from ``minicpmo-utils==1.0.6``, not installed and not vendored in the reference:
   ``engine/env/engine.lock:46``).  The classes carry the exact attribute names the engine reads
   (``engine/runtime/token2wav_batch.py:82-110,781-810``; ``engine/runtime/dit_fast.py:107-178``), so the reference's
   own driver (``BatchedToken2Wav._solve`` / ``_estimator_temb`` / ``_block_chunk`` / ``_conv_block_chunk``) runs
   unmodified on them; ``tests/golden/make_golden.py`` does exactly that to pin this oracle.
2. ``solve_packed``: the CFG Euler solve of packed ``[prompt | chunk]`` rows.  ``solve_window``: the steady-state form,
   one window of a stream against its estimator caches (keys ``[new, cache]``, two cached conv frames, the cache
   trimmed to the prompt's frames plus the last 100 after every kept window), as ``BatchedToken2Wav._solve`` and
   ``_flow_finish`` do it (``token2wav_batch.py:33-39,388-395,632-702``).  The reference solves the prompt alone
   first (``Flow.setup_cache``: all prompt frames attend each other, conv caches start at zero,
   ``token2wav_batch.py:551-553``) and then the chunk against the prompt's cached keys and conv frames of the same
   (step, block) (``token2wav_batch.py:632-702``).  The DiT has no positional encoding (``dit_fast.py:5-6``), so one
   sequence ``[prompt | chunk]`` with a block-causal mask (prompt queries see prompt keys; chunk queries see every key)
   and causal convolutions over the concatenation computes the same chunk mel.  The equivalence is checked against the
   reference's two-stage driver by ``tests/golden/make_golden.py``.

Parity pin: there is no published golden vector for this path (the reference's DiT tests need the checkpoint and a
GPU, ``tests/engine/test_dit_fast.py:16-17``).  The oracle is pinned against the reference's own solver code running on
these restated modules; fidelity of the restated modules to the real ``stepaudio2`` package is unpinned.
"""

from __future__ import annotations

import math
import os
import sys

import torch
import torch.nn as nn
import torch.nn.functional as F

_HERE = os.path.dirname(os.path.abspath(__file__))
_PKG = os.path.join(os.path.dirname(_HERE), "minicpm-o-4.5-single-gpu-engine_b200")
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

from b200t2w.config import DiTConfig, t_schedule  # noqa: E402


def modulate(x, shift, scale):
    """``decoder_dit.modulate`` as the engine uses it (``dit_kernels.py:27-28``): ``x * (1 + scale) + shift``."""
    return x * (1 + scale) + shift


class Transpose(nn.Module):
    def __init__(self, a: int, b: int):
        super().__init__()
        self.a, self.b = a, b

    def forward(self, x):
        return x.transpose(self.a, self.b)


class TimestepEmbedder(nn.Module):
    """Sinusoid of ``t * t_scale`` (cos half, then sin half) -> Linear -> SiLU -> Linear.  The frequency table is built
    on the host, as the reference's is (``dit_graph.py:40-41``)."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        self.cfg = cfg
        self.mlp = nn.Sequential(nn.Linear(cfg.freq_dim, cfg.hidden), nn.SiLU(), nn.Linear(cfg.hidden, cfg.hidden))

    def freq_embedding(self, t):
        half = self.cfg.freq_dim // 2
        freqs = torch.exp(-math.log(self.cfg.max_period) * torch.arange(half, dtype=torch.float32) / half).to(t.device)
        args = (t * self.cfg.t_scale)[:, None].float() * freqs[None]
        return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)

    def forward(self, t):
        return self.mlp(self.freq_embedding(t).to(self.mlp[0].weight.dtype))


class Attention(nn.Module):
    """``to_q/to_k/to_v`` (bias), per-head affine LayerNorm of q and k, SDPA (default scale), ``proj`` (bias)."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        inner = cfg.heads * cfg.head_dim
        self.num_heads, self.head_dim = cfg.heads, cfg.head_dim
        self.to_q = nn.Linear(cfg.hidden, inner)
        self.to_k = nn.Linear(cfg.hidden, inner)
        self.to_v = nn.Linear(cfg.hidden, inner)
        self.q_norm = nn.LayerNorm(cfg.head_dim, eps=cfg.eps_qk)
        self.k_norm = nn.LayerNorm(cfg.head_dim, eps=cfg.eps_qk)
        self.proj = nn.Linear(inner, cfg.hidden)

    def _heads(self, y):
        b, t, _ = y.shape
        return y.view(b, t, self.num_heads, self.head_dim).transpose(1, 2)

    def qkv(self, x):
        return self.q_norm(self._heads(self.to_q(x))), self.k_norm(self._heads(self.to_k(x))), self._heads(self.to_v(x))

    def attend(self, q, k, v, mask):
        b, _, t, _ = q.shape
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=None if mask is None else mask[:, None])
        return self.proj(o.transpose(1, 2).reshape(b, t, -1))

    def forward(self, x, mask=None):
        q, k, v = self.qkv(x)
        return self.attend(q, k, v, mask)

    def forward_chunk(self, x, att_cache=None, mask=None):
        """Keys/values are ``[new, cache]`` (the cache is appended after the window's frames); the new cache holds K
        (post-norm) and V concatenated on the last dim (``dit_fast.py:1-9``, ``token2wav_batch.py:696-698``)."""
        q, k, v = self.qkv(x)
        new = torch.cat([k, v], dim=-1)
        if att_cache is not None and att_cache.shape[2] > 0:
            new = torch.cat([new, att_cache.to(new.dtype)], dim=2)
        k, v = new.split(self.head_dim, dim=-1)
        return self.attend(q, k, v, mask), new


class CausalConv1d(nn.Conv1d):
    def __init__(self, cin: int, cout: int, k: int):
        super().__init__(cin, cout, k)
        self.causal_padding = (k - 1, 0)

    def forward(self, x):
        return super().forward(F.pad(x, self.causal_padding))


class CausalConvBlock(nn.Module):
    """``block = [T, CausalConv1d, T, LayerNorm(affine), Mish, T, CausalConv1d, T]`` (``token2wav_batch.py:90-97``)."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        H = cfg.hidden
        self.in_channels = self.out_channels = H
        self.block = nn.Sequential(Transpose(1, 2), CausalConv1d(H, H, cfg.conv_kernel), Transpose(1, 2),
                                   nn.LayerNorm(H, eps=cfg.eps_conv), nn.Mish(), Transpose(1, 2),
                                   CausalConv1d(H, H, cfg.conv_kernel), Transpose(1, 2))

    def forward(self, x):
        return self.block(x)


class Mlp(nn.Module):
    def __init__(self, cfg: DiTConfig):
        super().__init__()
        self.fc1 = nn.Linear(cfg.hidden, cfg.ffn)
        self.act = nn.GELU(approximate="tanh")
        self.fc2 = nn.Linear(cfg.ffn, cfg.hidden)

    def forward(self, x):
        return self.fc2(self.act(self.fc1(x)))


class DiTBlock(nn.Module):
    def __init__(self, cfg: DiTConfig):
        super().__init__()
        H = cfg.hidden
        self.norm1 = nn.LayerNorm(H, elementwise_affine=False, eps=cfg.eps_block)
        self.norm2 = nn.LayerNorm(H, elementwise_affine=False, eps=cfg.eps_block)
        self.norm3 = nn.LayerNorm(H, elementwise_affine=False, eps=cfg.eps_block)
        self.attn = Attention(cfg)
        self.conv = CausalConvBlock(cfg)
        self.mlp = Mlp(cfg)
        self.adaLN_modulation = nn.Sequential(nn.SiLU(), nn.Linear(H, 9 * H))

    def forward(self, x, c, mask):
        """Attention, conv, MLP with gated residuals; modulation chunk order fixed by ``token2wav_batch.py:104``."""
        sh_a, sc_a, g_a, sh_m, sc_m, g_m, sh_c, sc_c, g_c = self.adaLN_modulation(c).chunk(9, dim=-1)
        x = x + g_a * self.attn(modulate(self.norm1(x), sh_a, sc_a), mask)
        x = x + g_c * self.conv(modulate(self.norm3(x), sh_c, sc_c))
        return x + g_m * self.mlp(modulate(self.norm2(x), sh_m, sc_m))


class FinalLayer(nn.Module):
    def __init__(self, cfg: DiTConfig):
        super().__init__()
        self.norm_final = nn.LayerNorm(cfg.hidden, elementwise_affine=False, eps=cfg.eps_final)
        self.linear = nn.Linear(cfg.hidden, cfg.mel)
        self.adaLN_modulation = nn.Sequential(nn.SiLU(), nn.Linear(cfg.hidden, 2 * cfg.hidden))

    def forward(self, x, c):
        shift, scale = self.adaLN_modulation(c).chunk(2, dim=-1)
        return self.linear(modulate(self.norm_final(x), shift, scale))


class DiT(nn.Module):
    def __init__(self, cfg: DiTConfig):
        super().__init__()
        self.cfg = cfg
        self.out_channels = cfg.mel
        self.t_embedder = TimestepEmbedder(cfg)
        self.in_proj = nn.Linear(cfg.in_dim, cfg.hidden)
        self.blocks = nn.ModuleList([DiTBlock(cfg) for _ in range(cfg.depth)])
        self.final_layer = FinalLayer(cfg)

    def forward(self, x, mu, t, spks, cond, mask):
        """x, mu, cond [b, mel, L]; spks [b, mel]; t [b]; mask [b, L, L] bool (True: attend) -> dphi [b, mel, L]."""
        temb = self.t_embedder(t).unsqueeze(1)
        L = x.shape[2]
        h = self.in_proj(torch.cat([x, mu, spks[:, :, None].expand(-1, -1, L), cond], dim=1).transpose(1, 2))
        for blk in self.blocks:
            h = blk(h, temb, mask)
        return self.final_layer(h, temb).transpose(1, 2)


class CFM(nn.Module):
    """The ``CausalConditionalCFM`` attributes the engine reads: ``estimator``, ``inference_cfg_rate``, ``rand_noise``."""

    def __init__(self, cfg: DiTConfig, noise_frames: int = 2048):
        super().__init__()
        self.estimator = DiT(cfg)
        self.inference_cfg_rate = cfg.cfg_rate
        self.register_buffer("rand_noise", torch.zeros(1, cfg.mel, noise_frames))


def build_model(cfg: DiTConfig, seed: int = 0, noise_frames: int = 2048) -> CFM:
    """Random-init reference-config model.  ``torch.manual_seed(seed)`` then PyTorch's default Linear/Conv1d init in
    module construction order; every affine LayerNorm then gets weight ``1 + 0.1 N(0,1)`` and bias ``0.1 N(0,1)``; no
    zero-init of the adaLN or final layers (a zero-init DiT would make v == 0 and every parity test vacuous).  The
    noise buffer is drawn last."""
    torch.manual_seed(seed)
    m = CFM(cfg, noise_frames)
    with torch.no_grad():
        for mod in m.modules():
            if isinstance(mod, nn.LayerNorm) and mod.elementwise_affine:
                mod.weight.copy_(1 + 0.1 * torch.randn_like(mod.weight))
                mod.bias.copy_(0.1 * torch.randn_like(mod.bias))
        m.rand_noise.copy_(torch.randn_like(m.rand_noise))
    return m.eval()


def block_causal_mask(P: int, T: int) -> torch.Tensor:
    """[L, L] bool: prompt queries attend prompt keys only, chunk queries attend every key."""
    L = P + T
    lim = torch.where(torch.arange(L) < P, P, L)
    return torch.arange(L)[None, :] < lim[:, None]


@torch.inference_mode()
def solve_packed(model: CFM, x0, mu, cond, spk, P: int, T: int, dtype=torch.float32):
    """The full CFG Euler solve of ONE packed stream (``[prompt | chunk]``, L = P + T frames).

    x0, mu, cond: [mel, L] fp32; spk: [mel] (after the speaker affine layer).  Returns the final x [mel, L] fp32 (the
    chunk's mel is ``[:, P:]``).  Solver loop as ``token2wav_batch.py:666-694``: CFG rows ``[cond | uncond]`` with the
    uncond row's mu / spk / cond zeroed, ``x += dt * ((1 + w) * d - w * u)``, t accumulated."""
    est = model.estimator
    cfg = est.cfg
    w = float(model.inference_cfg_rate)
    L = P + T
    mask = block_causal_mask(P, T)[None].expand(2, -1, -1)
    x = x0.to(dtype)[None]
    mu_in = torch.stack([mu, torch.zeros_like(mu)]).to(dtype)
    spk_in = torch.stack([spk, torch.zeros_like(spk)]).to(dtype)
    cond_in = torch.stack([cond, torch.zeros_like(cond)]).to(dtype)
    ts, dts = t_schedule(cfg.steps)
    for t, dt in zip(ts, dts):
        v = est(x.expand(2, -1, -1), mu_in, torch.full((2,), t, dtype=torch.float32), spk_in, cond_in, mask)
        x = x + torch.tensor(dt, dtype=torch.float32) * ((1.0 + w) * v[0:1] - w * v[1:2])
    assert x.shape == (1, cfg.mel, L)
    return x[0].float()


def solve_streams(model: CFM, streams: list[dict], threads: int | None = None) -> list[torch.Tensor]:
    """``solve_packed`` for each stream dict (keys x0, mu, cond, spk, P, T); equal-shape streams are independent, so the
    oracle simply loops."""
    if threads:
        torch.set_num_threads(threads)
    return [solve_packed(model, s["x0"], s["mu"], s["cond"], s["spk"], s["P"], s["T"]) for s in streams]


TRIM_SUFFIX = 100


class StreamCache:
    """One request's estimator caches in the reference's layout (both CFG rows): ``att`` [S, depth, 2, heads, L,
    2 * head_dim] (K then V on the last dim, keys in ``[new, cache]`` order) and ``cnn`` [S, depth, 2, 2H, 2] (the two
    frames before the next window of each conv's input); ``keep`` is the trim length (the prompt's mel frames)."""

    def __init__(self, cfg: DiTConfig, keep: int = 0):
        self.att = torch.zeros(cfg.steps, cfg.depth, 2, cfg.heads, 0, 2 * cfg.head_dim)
        self.cnn = torch.zeros(cfg.steps, cfg.depth, 2, 2 * cfg.hidden, 2)
        self.keep = keep

    @property
    def length(self) -> int:
        return self.att.shape[4]


def trim(att: torch.Tensor, keep: int) -> torch.Tensor:
    """The reference's cache trim (``token2wav_batch.py:36-39``): over ``keep + 100`` keys, keep the first ``keep`` and
    the last 100."""
    L = att.shape[4]
    if L > keep + TRIM_SUFFIX:
        return torch.cat([att[:, :, :, :, :keep], att[:, :, :, :, L - TRIM_SUFFIX:]], dim=4)
    return att


def _conv_cached(conv: nn.Conv1d, x: torch.Tensor, cache: torch.Tensor):
    """A causal conv over ``[cached frames | window]``; returns (output [b, C, T], new cache = the last k - 1 frames)."""
    full = torch.cat([cache, x], dim=2)
    k1 = conv.kernel_size[0] - 1
    return F.conv1d(full, conv.weight, conv.bias), full[:, :, full.shape[2] - k1:]


@torch.inference_mode()
def solve_window(model: CFM, cache: StreamCache, x0, mu, spk, cond=None, keep_cache: bool = True) -> torch.Tensor:
    """One window of ``T`` frames of one stream: the CFG Euler solve against the stream's caches.

    x0, mu, cond: [mel, T] fp32 (cond None: zeros); spk: [mel].  Returns the window's mel [mel, T].  With
    ``keep_cache`` the caches become the window's new ones (keys ``[new, old]`` trimmed as the reference trims them,
    conv caches the last two input frames of each conv); otherwise (a final flush) they are left unchanged.  The
    caller takes x0 from the flow's fixed noise at the stream's cache length, as the reference does
    (``token2wav_batch.py:668``)."""
    est = model.estimator
    cfg = est.cfg
    w = float(model.inference_cfg_rate)
    H, T = cfg.hidden, x0.shape[1]
    x = x0.float()[None]
    mu_in = torch.stack([mu, torch.zeros_like(mu)]).float()
    spk_in = torch.stack([spk, torch.zeros_like(spk)]).float()
    c_in = torch.zeros_like(mu_in) if cond is None else torch.stack([cond, torch.zeros_like(cond)]).float()
    new_att, new_cnn = [], []
    ts, dts = t_schedule(cfg.steps)
    for step, (t, dt) in enumerate(zip(ts, dts)):
        temb = est.t_embedder(torch.full((2,), t, dtype=torch.float32)).unsqueeze(1)
        xx = x.expand(2, -1, -1)
        h = est.in_proj(torch.cat([xx, mu_in, spk_in[:, :, None].expand(-1, -1, T), c_in], dim=1).transpose(1, 2))
        att_s, cnn_s = [], []
        for b, blk in enumerate(est.blocks):
            sh_a, sc_a, g_a, sh_m, sc_m, g_m, sh_c, sc_c, g_c = blk.adaLN_modulation(temb).chunk(9, dim=-1)
            y, na = blk.attn.forward_chunk(modulate(blk.norm1(h), sh_a, sc_a), cache.att[step, b])
            h = h + g_a * y
            att_s.append(na)
            cb = blk.conv.block
            c1, c2 = cache.cnn[step, b].split(H, dim=1)
            a = modulate(blk.norm3(h), sh_c, sc_c).transpose(1, 2)
            y, n1 = _conv_cached(cb[1], a, c1)
            y = cb[4](cb[3](y.transpose(1, 2))).transpose(1, 2)
            y, n2 = _conv_cached(cb[6], y, c2)
            h = h + g_c * y.transpose(1, 2)
            cnn_s.append(torch.cat([n1, n2], dim=1))
            h = h + g_m * blk.mlp(modulate(blk.norm2(h), sh_m, sc_m))
        v = est.final_layer(h, temb).transpose(1, 2)
        x = x + torch.tensor(dt, dtype=torch.float32) * ((1.0 + w) * v[0:1] - w * v[1:2])
        new_att.append(torch.stack(att_s))
        new_cnn.append(torch.stack(cnn_s))
    if keep_cache:
        cache.att = trim(torch.stack(new_att), cache.keep)
        cache.cnn = torch.stack(new_cnn)
    return x[0].float()


def state_dict_np(model: CFM) -> dict:
    """fp32 weights keyed by the reference module paths (``estimator.blocks.3.attn.to_q.weight`` ...)."""
    return {k: v.detach().float().contiguous() for k, v in model.state_dict().items() if k != "rand_noise"}
