"""Random-init weights of the reference DiT architecture, generated directly as a state dict (no module objects).

PyTorch's default init for the reference's ``nn.Linear`` / ``nn.Conv1d`` layers draws weight and bias from
U(-1/sqrt(fan_in), 1/sqrt(fan_in)); affine LayerNorms get weight 1 + 0.1 N(0,1) and bias 0.1 N(0,1), and nothing is
zero-initialised (a zero-init adaLN / final layer would make the velocity identically zero).  Keys are the
``estimator.<path>`` names the solver binds (``b200t2w.lib.W_GLOBAL`` / ``W_BLOCK``).  The values are drawn from a
seeded generator on the target device, so large configs are generated in milliseconds; they are not the same draws as
a module built under ``torch.manual_seed`` (parity tests bind the oracle module's own weights instead).
"""

from __future__ import annotations

import math

import torch

from .config import DiTConfig


def random_state_dict(cfg: DiTConfig, seed: int = 0, device="cpu") -> dict:
    g = torch.Generator(device=device).manual_seed(seed)
    H, F, D, mel = cfg.hidden, cfg.ffn, cfg.head_dim, cfg.mel
    out: dict = {}

    def lin(name: str, n_out: int, fan_in: int, shape=None):
        b = 1.0 / math.sqrt(fan_in)
        out[name + ".weight"] = (torch.rand(shape or (n_out, fan_in), generator=g, device=device) * 2 - 1) * b
        out[name + ".bias"] = (torch.rand(n_out, generator=g, device=device) * 2 - 1) * b

    def ln(name: str, n: int):
        out[name + ".weight"] = 1 + 0.1 * torch.randn(n, generator=g, device=device)
        out[name + ".bias"] = 0.1 * torch.randn(n, generator=g, device=device)

    e = "estimator."
    lin(e + "t_embedder.mlp.0", H, cfg.freq_dim)
    lin(e + "t_embedder.mlp.2", H, H)
    lin(e + "in_proj", H, cfg.in_dim)
    for b in range(cfg.depth):
        p = f"{e}blocks.{b}."
        lin(p + "attn.to_q", H, H)
        lin(p + "attn.to_k", H, H)
        lin(p + "attn.to_v", H, H)
        ln(p + "attn.q_norm", D)
        ln(p + "attn.k_norm", D)
        lin(p + "attn.proj", H, H)
        lin(p + "conv.block.1", H, H * cfg.conv_kernel, shape=(H, H, cfg.conv_kernel))
        ln(p + "conv.block.3", H)
        lin(p + "conv.block.6", H, H * cfg.conv_kernel, shape=(H, H, cfg.conv_kernel))
        lin(p + "mlp.fc1", F, H)
        lin(p + "mlp.fc2", H, F)
        lin(p + "adaLN_modulation.1", 9 * H, H)
    lin(e + "final_layer.linear", mel, H)
    lin(e + "final_layer.adaLN_modulation.1", 2 * H, H)
    return out
