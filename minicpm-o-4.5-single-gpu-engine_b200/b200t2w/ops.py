"""The torch custom ops ``torch.ops.b200t2w.*`` (``libt2w_torch_ops.so``, a thin shim over the C ABI of
``libt2w_b200.so``; schemas in ``csrc/torch_ops.cpp``).

The solver classes call their solves through these ops, so the engine's torch code (``BatchedToken2Wav`` calling
``FastDiT.solve``: ``engine/runtime/token2wav_batch.py:335,356-357,518-519,549``) sees registered operators that run on
the current torch stream.  There is no fallback: if the shim is missing, ``load()`` raises.  A failing op raises
``RuntimeError("t2w_... failed: status N ...")``; ``call`` turns that into ``T2WError`` with the same status as the
ctypes binding.
"""

from __future__ import annotations

import os
import re

import torch

from . import lib as L
from .build import OPS_PATH

_loaded = False


def load(path: str | None = None):
    """Register the ops (once) and return the ``torch.ops.b200t2w`` namespace."""
    global _loaded
    if not _loaded:
        path = path or OPS_PATH
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with b200t2w.build.build_ops()")
        L.load()  # the C library first, by its path (the shim finds it by soname)
        torch.ops.load_library(path)
        _loaded = True
    return torch.ops.b200t2w


def call(name: str, *args):
    """``torch.ops.b200t2w.<name>(*args)``, with a failed status raised as ``T2WError``."""
    op = getattr(load(), name)
    try:
        return op(*args)
    except RuntimeError as e:
        m = re.search(r"(t2w_\w+) failed: status (-?\d+)(?: \(cudaError (\d+)\))?", str(e))
        if not m:
            raise
        raise L.T2WError(m.group(1), int(m.group(2)), int(m.group(3) or 0)) from e


OPS = ("create", "destroy", "workspace_bytes", "solve_packed", "slots_create", "slots_destroy", "cached_workspace_bytes",
       "solve_cached", "solve_slots", "ln_mod", "add_ln_mod", "ln_mish", "gemm", "attn_varlen", "euler_cfg",
       "enc_workspace_bytes", "encode")
