"""Host logic of the HiFT vocoder binding: the ``decode_tf32`` values (True / False / lists of stages and
``"<stage>:<part>"`` entries, as the reference's ``tf32_stages`` reads them, engine/models/token2wav.py:145-158) mapped to
the library's per-part mask (bit 3 s + p; parts ups, src, res)."""

import pytest

from b200t2w.hift import PARTS, tf32_parts


def test_all_and_none():
    assert tf32_parts(True) == 0x1FF
    for v in (False, None, [], ()):
        assert tf32_parts(v) == 0


def test_stage_and_part_entries():
    assert tf32_parts([0]) == 0b111
    assert tf32_parts([2]) == 0b111 << 6
    assert tf32_parts(["1:src"]) == 1 << 4
    # the reference's documented served combination: stage 0's transposed convolution stays fp32
    assert tf32_parts([1, 2, "0:src", "0:res"]) == 0x1FF & ~1
    assert tf32_parts(["0:ups", "0:src", "0:res", 1, 2]) == 0x1FF
    assert PARTS == ("ups", "src", "res")


@pytest.mark.parametrize("bad", [[3], ["-1"], ["0:conv"], ["x"]])
def test_rejects_unknown_entries(bad):
    with pytest.raises((ValueError, AssertionError)):
        tf32_parts(bad)


def test_decode_tf32_config_to_vocoder_mode():
    """``B200HiFT.for_decode_tf32``: the reference's default (False / None, strict fp32) maps to the split-form fp32
    mode on the tensor cores, True and stage lists to the same TF32 parts (checked without a GPU: the constructor's
    arguments are recorded)."""
    import torch

    from b200t2w.hift import B200HiFT

    calls = []

    class Rec(B200HiFT):
        def __init__(self, cfg, weights, **kw):
            calls.append(kw)

        def __del__(self):
            pass

    m = torch.nn.Linear(2, 2)
    for v in (False, None, True, [1, "0:src"]):
        Rec.for_decode_tf32(m, v)
    assert calls == [{"split_fp32": True}, {"split_fp32": True}, {"tf32": True}, {"tf32": [1, "0:src"]}]
