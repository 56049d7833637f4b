"""CPU: the C-ABI library builds, loads without a GPU driver, and exports every function ``include/*.h`` declares; the
host-side tables agree with the header.  No compute call is made here."""

import ctypes
import os
import re

import torch

from b200t2w import lib as L
from b200t2w.build import INCLUDE, build


def test_library_exports_every_header_symbol():
    path = build()
    so = ctypes.CDLL(path)
    syms = L.header_symbols()
    assert len(syms) >= 15, syms
    missing = [s for s in syms if not hasattr(so, s)]
    assert not missing, missing
    assert set(syms) <= set(L._SIGS), set(syms) - set(L._SIGS)


def test_version_and_device_probe():
    lib = L.load()
    assert lib.t2w_version() == 1
    if not torch.cuda.is_available():
        assert lib.t2w_device_ok(0) == 0


def _enum_len(src: str, name: str) -> int:
    body = re.search(r"enum\s+" + name + r"\s*\{(.*?)\};", src, flags=re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    return len([t for t in body.replace("\n", " ").split(",") if t.strip() and "COUNT" not in t])


def test_weight_slots_match_header():
    src = open(os.path.join(INCLUDE, "t2w_b200.h")).read()
    assert _enum_len(src, "t2w_weight_slot") == len(L.W_GLOBAL)
    assert _enum_len(src, "t2w_block_slot") == len(L.W_BLOCK)


def test_weight_names_exist_in_the_estimator_layout():
    from b200t2w.config import TINY
    from oracle import dit_oracle

    sd = {f"estimator.{k}" for k in dit_oracle.build_model(TINY).estimator.state_dict()}
    names = L.W_GLOBAL + [f"estimator.blocks.{b}.{n}" for b in range(TINY.depth) for n in L.W_BLOCK]
    assert set(names) <= sd, set(names) - sd
    # every parameter the kernels need is bound (nothing silently dropped)
    assert sd - set(names) == set()


def test_error_status_is_an_exception():
    e = L.T2WError("t2w_solve_packed", -6)
    assert "workspace" in str(e) and e.status == -6


def test_varlen_attention_rejects_overflowing_rows_without_a_gpu():
    """A sequence whose end (seq_row + seq_len) passes INT32_MAX is refused by the size check, which is computed in
    64 bits and comes before any CUDA call (no device is touched; the pointers are never read)."""
    for fn in ("t2w_attn_varlen", "t2w_attn_varlen_noalloc"):
        rc = getattr(L.load(), fn)(ctypes.c_void_p(16), 1000, 1, 1, L.i32_array([2**31 - 10]), L.i32_array([100]),
                                   L.i32_array([100]), ctypes.c_void_p(16), None)
        assert rc == -1, (fn, rc)


def test_torch_ops_are_registered():
    """The torch custom-op shim builds, loads without a GPU, and registers every op over the C ABI."""
    from b200t2w import ops
    from b200t2w.build import build_ops

    ns = ops.load(build_ops())
    for name in ops.OPS:
        assert hasattr(ns, name), name
    schema = str(ns.solve_packed.default._schema)
    assert schema.startswith("b200t2w::solve_packed(int solver, int[] prompt_len, int[] chunk_len"), schema
    assert "Tensor(a!) out" in schema


def test_torch_op_error_is_a_t2w_error_without_a_gpu():
    """A failing op's status crosses torch's dispatcher as an exception (the shim shares torch's C++ runtime) and
    comes back as ``T2WError``: destroying a null solver is refused before any CUDA call."""
    import pytest

    from b200t2w import ops

    with pytest.raises(L.T2WError) as e:
        ops.call("destroy", 0)
    assert e.value.status == -1
