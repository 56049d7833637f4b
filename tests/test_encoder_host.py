"""CPU: the flow encoder's host side — config read off a flow module, and the weight-slot tables the ctypes binding
hands to ``t2w_encoder_create`` against the header's enums and the flow module's state-dict paths."""

import os
import re

import pytest

from b200t2w import lib as L
from b200t2w.config import ENCODER, ENCODER_TINY
from b200t2w.encoder import encoder_config_from_flow
from oracle import encoder_oracle as eo


@pytest.mark.parametrize("cfg", [ENCODER_TINY, ENCODER])
def test_config_from_flow(cfg):
    assert encoder_config_from_flow(eo.build_flow(cfg, seed=0)) == cfg


def _enum_names(src: str, enum: str) -> list:
    body = re.search(r"enum " + enum + r"\s*\{(.*?)\};", src, flags=re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    return [n.split("=")[0].strip() for n in body.split(",") if n.strip()]


def test_weight_slots_match_header_and_module():
    src = open(os.path.join(L.INCLUDE, "t2w_b200.h")).read()
    g = _enum_names(src, "t2w_enc_weight_slot")
    y = _enum_names(src, "t2w_enc_layer_slot")
    assert g[-1] == "T2W_E_COUNT" and y[-1] == "T2W_EL_COUNT"
    assert len(L.E_GLOBAL) == len(g) - 1 and len(L.E_LAYER) == len(y) - 1
    sd = eo.build_flow(ENCODER_TINY, seed=0).state_dict()
    for n in L.E_GLOBAL:
        assert n in sd, n
    for p in ("encoder.encoders.0.", "encoder.up_encoders.1."):
        for n in L.E_LAYER:
            assert p + n in sd, p + n


def test_enc_structs_match_header():
    src = open(os.path.join(L.INCLUDE, "t2w_b200.h")).read()
    body = re.search(r"typedef struct t2w_enc_config \{(.*?)\} t2w_enc_config;", src, flags=re.S).group(1)
    fields = re.findall(r"(\w+)(?=[,;])", body)
    assert fields == [f for f, _ in L.EncConfig._fields_]
