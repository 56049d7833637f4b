"""CPU: the config read off a loaded CFM module, as the reference's ``FastDiT`` reads it
(``engine/runtime/dit_fast.py:107-145``), and ``B200FastDiT.from_cfm``'s argument checks (made before any device work)."""

import pytest
import torch

from b200t2w.config import REFERENCE, TINY, config_from_module
from b200t2w.fastdit import B200FastDiT
from oracle import dit_oracle


@pytest.mark.parametrize("cfg", [TINY, REFERENCE], ids=["tiny", "reference"])
def test_config_round_trip(cfg):
    m = dit_oracle.build_model(cfg, seed=0, noise_frames=16)
    assert config_from_module(m, steps=cfg.steps) == cfg


def test_config_reads_module_not_defaults():
    """Every field the module carries comes from the module, not from the base config."""
    m = dit_oracle.build_model(TINY, seed=0, noise_frames=16)
    m.inference_cfg_rate = 0.5
    for blk in m.estimator.blocks:
        blk.attn.q_norm.eps = blk.attn.k_norm.eps = 1e-4
        blk.conv.block[3].eps = 2e-5
    m.estimator.final_layer.norm_final.eps = 3e-6
    c = config_from_module(m, steps=4)
    assert (c.cfg_rate, c.eps_qk, c.eps_conv, c.eps_final, c.steps) == (0.5, 1e-4, 2e-5, 3e-6, 4)
    assert (c.hidden, c.depth, c.heads, c.head_dim, c.ffn, c.mel) == (128, 2, 2, 64, 512, 80)


def test_config_rejects_inconsistent_module():
    m = dit_oracle.build_model(TINY, seed=0, noise_frames=16)
    m.estimator.blocks[0].attn.k_norm.eps = 1e-3
    with pytest.raises(ValueError, match="q_norm"):
        config_from_module(m)
    m = dit_oracle.build_model(TINY, seed=0, noise_frames=16)
    m.estimator.blocks[0].norm2.eps = 1e-5
    with pytest.raises(ValueError, match="norm1"):
        config_from_module(m)
    m = dit_oracle.build_model(TINY, seed=0, noise_frames=16)
    m.estimator.in_proj = torch.nn.Linear(4 * TINY.mel + 1, TINY.hidden)
    with pytest.raises(ValueError, match="in_proj"):
        config_from_module(m)


def test_from_cfm_option_checks():
    m = dit_oracle.build_model(TINY, seed=0, noise_frames=16)
    with pytest.raises(ValueError, match="fused_residual"):
        B200FastDiT.from_cfm(m, TINY.steps, fused_conv=True)
    with pytest.raises(ValueError, match="setup_tokens"):
        B200FastDiT.from_cfm(m, TINY.steps, setup_tokens=-1)
