"""CPU fp32 oracle of the Token2Wav flow encoder's chunk forward.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this module, and only as
the checker: the product (the ``b200t2w`` package and its CUDA library) never calls into it.

1. A restatement of the third-party modules the reference engine drives for the flow encoder
   (``stepaudio2.cosyvoice2.transformer.upsample_encoder.UpsampleConformerEncoderV2`` and the flow's
   ``input_embedding`` / ``encoder_proj`` / ``spk_embed_affine_layer``, from ``minicpmo-utils==1.0.6``, absent here:
   ``engine/env/engine.lock:46``).  The classes carry the attribute names and call forms the engine uses
   (``engine/runtime/token2wav_batch.py:42-79,363-371,402-478,556-616``): ``enc.embed(xs, None)`` and
   ``enc.embed.position_encoding(offset, size)``, ``enc.pre_lookahead_layer.forward_chunk(xs, cache)`` with ``conv1`` /
   ``conv2`` / ``pre_lookahead_len``, ``layer(xs, mask, pos, att_cache=...)`` returning ``(xs, mask, new_att_cache,
   new_cnn_cache)``, ``enc.up_layer.forward_chunk(xs, lens, cache)`` with ``conv`` / ``stride`` / ``scale_factor``,
   ``enc.up_embed``, ``enc.up_encoders``, ``enc.normalize_before``, ``enc.after_norm``, and ``enc.forward_chunk(xs,
   last_chunk, cnn_cache, att_cache)``.  The arithmetic follows the published ESPnet / WeNet / CosyVoice2 algorithms:
   linear input layer (Linear, LayerNorm, times sqrt(d)); relative positional encoding ``pe(r) = [sin r w_m, cos r
   w_m]`` over r = size - 1 .. -(size - 1); relative-position self-attention with ``pos_bias_u`` / ``pos_bias_v`` and the
   zero-pad ``rel_shift``; pre-norm conformer layers without conv module or macaron feed-forward (swish FFN); a
   pre-lookahead layer (a look-ahead conv, leaky ReLU, a causal 3-tap conv, residual); nearest x2 upsampling followed
   by a causal 5-tap conv.  Its fidelity to the real package is unpinned (the package is absent).
2. The batched chunk forward as the engine runs it, pinned by ``tests/golden/make_encoder_golden.py``, which runs the
   reference's own ``BatchedToken2Wav._setup_encoder_batched`` / ``_encoder`` / ``_flow_finish`` (left-padded caches,
   masks, trims) on these modules.  ``EncoderStream`` + ``encode_window`` restate that per stream, unpadded:
   ``encode_prompt`` (prompt tokens plus 3 silence tokens, empty caches) and ``encode_window`` (a window against the
   stream's caches; keeps the trim rule of ``_flow_finish``: the attention cache ``[c1, c1, c2]`` along time is cut to its
   first ``keep`` and last 100 frames, and the first stack then reads the first half of that cut).
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

from b200t2w.config import EncoderConfig  # noqa: E402

TRIM_SUFFIX = 100
SILENCE_TOKEN = 4218  # engine/models/token2wav.py:39


class RelPositionalEncoding(nn.Module):
    """ESPnet relative positional encoding: ``position_encoding(offset, size)`` -> [1, 2 size - 1, d], row k holding
    ``pe(size - 1 - k)``; calling it scales ``x`` by sqrt(d) and returns the encoding for ``x``'s length."""

    def __init__(self, d: int, max_period: float = 10000.0):
        super().__init__()
        self.d, self.max_period = d, max_period
        self.xscale = math.sqrt(d)
        # follows the module's device and dtype (.to / .half), as the encoding buffer of the real module does
        self.register_buffer("anchor", torch.zeros(0), persistent=False)

    def position_encoding(self, offset, size: int) -> torch.Tensor:
        r = torch.arange(size - 1, -size, -1, dtype=torch.float32)[:, None]
        w = torch.exp(torch.arange(0, self.d, 2, dtype=torch.float32) * -(math.log(self.max_period) / self.d))
        pe = torch.zeros(2 * size - 1, self.d)
        pe[:, 0::2] = torch.sin(r * w)
        pe[:, 1::2] = torch.cos(r * w)
        return pe[None].to(self.anchor.device, self.anchor.dtype)

    def forward(self, x: torch.Tensor, offset=0):
        return x * self.xscale, self.position_encoding(offset, x.shape[1])


class LinearNoSubsampling(nn.Module):
    """Linear input layer: Linear, LayerNorm, then the positional encoding's sqrt(d) scale."""

    def __init__(self, idim: int, odim: int, eps: float, max_period: float):
        super().__init__()
        self.out = nn.Sequential(nn.Linear(idim, odim), nn.LayerNorm(odim, eps=eps))
        self.pos_enc = RelPositionalEncoding(odim, max_period)

    def position_encoding(self, offset, size: int) -> torch.Tensor:
        return self.pos_enc.position_encoding(offset, size)

    def forward(self, x, x_mask, offset=0):
        x, pos = self.pos_enc(self.out(x), offset)
        return x, pos, x_mask


class RelPositionAttention(nn.Module):
    """Multi-head self-attention with relative positions (Transformer-XL form, ESPnet ``rel_shift``)."""

    def __init__(self, heads: int, d: int):
        super().__init__()
        self.h, self.d_k = heads, d // heads
        self.linear_q, self.linear_k, self.linear_v = nn.Linear(d, d), nn.Linear(d, d), nn.Linear(d, d)
        self.linear_out = nn.Linear(d, d)
        self.linear_pos = nn.Linear(d, d, bias=False)
        self.pos_bias_u = nn.Parameter(torch.empty(heads, self.d_k))
        self.pos_bias_v = nn.Parameter(torch.empty(heads, self.d_k))
        nn.init.xavier_uniform_(self.pos_bias_u)
        nn.init.xavier_uniform_(self.pos_bias_v)

    @staticmethod
    def rel_shift(x: torch.Tensor) -> torch.Tensor:
        """[b, h, T, 2K - 1] -> [b, h, T, K]: a zero column in front, the rows re-read with one more column each, so
        query i's column j reads its input column ``j + T - 1 - i`` (relative position ``K - T + i - j``)."""
        b, h, t, p = x.shape
        xp = torch.cat([x.new_zeros(b, h, t, 1), x], dim=-1).view(b, h, p + 1, t)
        return xp[:, :, 1:].reshape(b, h, t, p)[:, :, :, : p // 2 + 1]

    def forward(self, x: torch.Tensor, mask: torch.Tensor, pos: torch.Tensor, cache: torch.Tensor):
        b, t, _ = x.shape
        q = self.linear_q(x).view(b, t, self.h, self.d_k)
        k = self.linear_k(x).view(b, t, self.h, self.d_k).transpose(1, 2)
        v = self.linear_v(x).view(b, t, self.h, self.d_k).transpose(1, 2)
        if cache is not None and cache.shape[0] > 0:
            kc, vc = cache.split(self.d_k, dim=-1)
            k, v = torch.cat([kc, k], dim=2), torch.cat([vc, v], dim=2)
        new_cache = torch.cat([k, v], dim=-1)
        p = self.linear_pos(pos).view(pos.shape[0], -1, self.h, self.d_k).transpose(1, 2)
        ac = torch.matmul((q + self.pos_bias_u).transpose(1, 2), k.transpose(-2, -1))
        bd = torch.matmul((q + self.pos_bias_v).transpose(1, 2), p.transpose(-2, -1))
        if bd.shape != ac.shape:
            bd = self.rel_shift(bd)
        scores = (ac + bd) / math.sqrt(self.d_k)
        keep = mask[:, None, :, : scores.shape[-1]].bool()
        scores = scores.masked_fill(~keep, -float("inf"))
        attn = torch.softmax(scores, dim=-1).masked_fill(~keep, 0.0)
        out = torch.matmul(attn, v).transpose(1, 2).reshape(b, t, -1)
        return self.linear_out(out), new_cache


class FeedForward(nn.Module):
    def __init__(self, d: int, hidden: int):
        super().__init__()
        self.w_1, self.w_2 = nn.Linear(d, hidden), nn.Linear(hidden, d)

    def forward(self, x):
        return self.w_2(F.silu(self.w_1(x)))


class ConformerLayer(nn.Module):
    """Pre-norm layer: ``x + attn(norm_mha(x))`` then ``x + ff(norm_ff(x))``; returns (x, mask, new att cache, cnn)."""

    def __init__(self, cfg: EncoderConfig):
        super().__init__()
        self.self_attn = RelPositionAttention(cfg.heads, cfg.hidden)
        self.feed_forward = FeedForward(cfg.hidden, cfg.ffn)
        self.norm_mha = nn.LayerNorm(cfg.hidden, eps=cfg.eps_layer)
        self.norm_ff = nn.LayerNorm(cfg.hidden, eps=cfg.eps_layer)

    def forward(self, x, mask, pos_emb, mask_pad=None, att_cache=None, cnn_cache=None):
        a, new_cache = self.self_attn(self.norm_mha(x), mask, pos_emb, att_cache)
        x = x + a
        x = x + self.feed_forward(self.norm_ff(x))
        return x, mask, new_cache, torch.zeros(0)


class PreLookaheadLayer(nn.Module):
    """conv1 over each frame and its ``pre_lookahead_len`` successors, leaky ReLU, a causal 3-tap conv2 (2 cached
    frames of conv1's output), plus the input."""

    def __init__(self, cfg: EncoderConfig):
        super().__init__()
        self.pre_lookahead_len = cfg.lookahead
        self.slope = cfg.leaky_slope
        self.conv1 = nn.Conv1d(cfg.hidden, cfg.hidden, cfg.lookahead + 1)
        self.conv2 = nn.Conv1d(cfg.hidden, cfg.hidden, 3)

    def forward_chunk(self, xs: torch.Tensor, cache: torch.Tensor | None = None):
        """xs [b, T + lookahead, c] -> ([b, T, c], new cache [b, c, 2]: conv1's last two output frames)."""
        o = F.leaky_relu(self.conv1(xs.transpose(1, 2)), self.slope)
        if cache is None or cache.shape[-1] == 0:
            cache = o.new_zeros(o.shape[0], o.shape[1], 2)
        new_cache = o[:, :, -2:]
        o = self.conv2(torch.cat([cache, o], dim=2))
        return o.transpose(1, 2) + xs[:, : o.shape[2]], new_cache


class Upsample1D(nn.Module):
    """Nearest upsampling by ``stride`` then a causal ``2 stride + 1``-tap conv (``2 stride`` cached frames)."""

    def __init__(self, cfg: EncoderConfig):
        super().__init__()
        self.stride = cfg.stride
        self.scale_factor = float(cfg.stride)
        self.conv = nn.Conv1d(cfg.hidden, cfg.hidden, 2 * cfg.stride + 1)

    def forward_chunk(self, xs: torch.Tensor, lens, cache: torch.Tensor | None = None):
        """xs [b, c, T] -> ([b, c, stride T], lens, new cache [b, c, 2 stride])."""
        u = F.interpolate(xs, scale_factor=self.scale_factor, mode="nearest")
        if cache is None or cache.shape[-1] == 0:
            cache = u.new_zeros(u.shape[0], u.shape[1], 2 * self.stride)
        u = torch.cat([cache, u], dim=2)
        return self.conv(u), lens, u[:, :, -2 * self.stride:]


class UpsampleConformerEncoder(nn.Module):
    def __init__(self, cfg: EncoderConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = LinearNoSubsampling(cfg.hidden, cfg.hidden, cfg.eps_embed, cfg.max_period)
        self.pre_lookahead_layer = PreLookaheadLayer(cfg)
        self.encoders = nn.ModuleList([ConformerLayer(cfg) for _ in range(cfg.blocks1)])
        self.up_layer = Upsample1D(cfg)
        self.up_embed = LinearNoSubsampling(cfg.hidden, cfg.hidden, cfg.eps_embed, cfg.max_period)
        self.up_encoders = nn.ModuleList([ConformerLayer(cfg) for _ in range(cfg.blocks2)])
        self.normalize_before = True
        self.after_norm = nn.LayerNorm(cfg.hidden, eps=cfg.eps_after)

    def forward_chunk(self, xs, last_chunk: bool = False, cnn_cache=None, att_cache=None):
        """One stream (batch 1): xs [1, tokens, c] embedded tokens (with ``lookahead`` look-ahead tokens unless
        ``last_chunk``); caches as the engine keeps them (cnn [1, c, 2 + 2 stride], att [d1 + d2, 1, nh, 2 t, 2 d_k]
        with the first stack's t frames tiled twice).  Returns (xs [1, stride T, c] after ``after_norm``, new cnn
        cache, new att cache in the same layout)."""
        cfg = self.cfg
        d1, s = cfg.blocks1, cfg.stride
        t1 = 0 if att_cache is None else att_cache.shape[3] // 2
        xs, _, _ = self.embed(xs, None)
        if last_chunk:
            xs = F.pad(xs, (0, 0, 0, cfg.lookahead))
        c1 = None if cnn_cache is None else cnn_cache[:, :, :2]
        c2 = None if cnn_cache is None else cnn_cache[:, :, 2:]
        xs, n1 = self.pre_lookahead_layer.forward_chunk(xs, c1)
        T = xs.shape[1]
        mask = torch.ones(1, T, t1 + T, dtype=torch.bool)
        pos = self.embed.position_encoding(None, t1 + T)
        new1 = []
        for i, layer in enumerate(self.encoders):
            ac = None if att_cache is None else att_cache[i, :, :, :t1]
            xs, _, c, _ = layer(xs, mask, pos, att_cache=ac)
            new1.append(c)
        xs, _, n2 = self.up_layer.forward_chunk(xs.transpose(1, 2), None, c2)
        xs, _, _ = self.up_embed(xs.transpose(1, 2), None)
        mask = torch.ones(1, s * T, s * (t1 + T), dtype=torch.bool)
        pos = self.embed.position_encoding(None, s * (t1 + T))
        new2 = []
        for i, layer in enumerate(self.up_encoders):
            ac = None if att_cache is None else att_cache[d1 + i]
            xs, _, c, _ = layer(xs, mask, pos, att_cache=ac)
            new2.append(c)
        xs = self.after_norm(xs)
        att = torch.cat([torch.stack(new1).repeat(1, 1, 1, 2, 1), torch.stack(new2)], dim=0)
        return xs, torch.cat([n1, n2], dim=2), att


class Flow(nn.Module):
    """The flow-module pieces around the encoder: token embedding, encoder, ``encoder_proj`` (-> mu channels) and the
    speaker affine layer."""

    def __init__(self, cfg: EncoderConfig):
        super().__init__()
        self.cfg = cfg
        self.input_embedding = nn.Embedding(cfg.vocab, cfg.hidden)
        self.encoder = UpsampleConformerEncoder(cfg)
        self.encoder_proj = nn.Linear(cfg.hidden, cfg.mel)
        self.spk_embed_affine_layer = nn.Linear(cfg.spk_dim, cfg.mel)


def build_flow(cfg: EncoderConfig, seed: int = 0) -> Flow:
    """Random-init flow encoder.  ``torch.manual_seed(seed)``, PyTorch's default init in construction order, then
    every affine LayerNorm gets weight ``1 + 0.1 N(0,1)`` and bias ``0.1 N(0,1)`` and the embedding table is scaled by
    0.5 (activations of order one through the stacks)."""
    torch.manual_seed(seed)
    m = Flow(cfg)
    with torch.no_grad():
        for mod in m.modules():
            if isinstance(mod, nn.LayerNorm):
                mod.weight.copy_(1 + 0.1 * torch.randn_like(mod.weight))
                mod.bias.copy_(0.1 * torch.randn_like(mod.bias))
        m.input_embedding.weight.mul_(0.5)
    return m.eval()


def trim_att(att: torch.Tensor, keep: int) -> torch.Tensor:
    """``_trim(att, keep, 3)`` (``token2wav_batch.py:36-39``)."""
    if att.shape[3] > keep + TRIM_SUFFIX:
        return torch.cat([att[:, :, :, :keep], att[:, :, :, att.shape[3] - TRIM_SUFFIX:]], dim=3)
    return att


class EncoderStream:
    """One stream's flow-encoder state as the engine keeps it: ``cnn`` [1, c, 2 + 2 stride], ``att`` [d1 + d2, 1, nh,
    2 t, 2 d_k] and the trim length ``keep`` (the prompt's mel frames)."""

    def __init__(self, cnn: torch.Tensor, att: torch.Tensor, keep: int):
        self.cnn, self.att, self.keep = cnn, att, keep


@torch.no_grad()
def encode_prompt(flow: Flow, tokens: torch.Tensor) -> tuple[torch.Tensor, EncoderStream]:
    """A prompt's setup (``_setup_encoder_one``, ``token2wav_batch.py:556-564``): its tokens plus ``lookahead`` silence
    tokens through ``forward_chunk`` with empty caches.  Returns (mu [mel, 2 n] = ``encoder_proj`` output transposed, the
    stream), keep = 2 n."""
    cfg = flow.cfg
    toks = torch.cat([tokens.reshape(1, -1), torch.full((1, cfg.lookahead), SILENCE_TOKEN, dtype=tokens.dtype)], 1)
    h, cnn, att = flow.encoder.forward_chunk(flow.input_embedding(toks), last_chunk=False)
    mu = flow.encoder_proj(h)[0].t().contiguous()
    return mu, EncoderStream(cnn.clone(), att.clone(), int(mu.shape[1]))


@torch.no_grad()
def encode_window(flow: Flow, st: EncoderStream, tokens: torch.Tensor, last: bool) -> torch.Tensor:
    """One window (``_flow_encode`` + ``_encoder`` + ``_flow_finish`` for one stream): ``tokens`` [n] (with the look-ahead
    tokens unless ``last``) against the stream's caches; the caches advance and the attention cache is trimmed (a final
    window's caches are never read again but advance the same way).  Returns mu [mel, stride T]."""
    h, cnn, att = flow.encoder.forward_chunk(flow.input_embedding(tokens.reshape(1, -1)), last_chunk=last,
                                             cnn_cache=st.cnn, att_cache=st.att)
    st.cnn, st.att = cnn, trim_att(att, st.keep)
    return flow.encoder_proj(h)[0].t().contiguous()


def state_dict_np(flow: Flow) -> dict:
    return {k: v.detach().float().numpy() for k, v in flow.state_dict().items()}
