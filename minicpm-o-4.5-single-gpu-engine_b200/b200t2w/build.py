"""Build recipe of ``libt2w_b200.so``: the sm_100a CUDA kernels and the C ABI, compiled in-tree with nvcc.

``python -m b200t2w.build`` (or ``build()``) compiles every ``csrc/*.cu`` to an object with
``-gencode arch=compute_100a,code=sm_100a -lineinfo`` and links them into ``<package>/lib/libt2w_b200.so``.  The CUDA
runtime is linked statically and the driver API is reached through ``cudaGetDriverEntryPoint``, so the library loads on
a machine without a GPU driver (nothing computes there).  Objects are rebuilt only when a source or header is newer.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPO = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_DIR = os.path.join(PKG_ROOT, "lib")
OBJ_DIR = os.path.join(PKG_ROOT, "_build")
LIB_PATH = os.path.join(LIB_DIR, "libt2w_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "-Xptxas", "-warn-spills", "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]


def build(verbose: bool = False, force: bool = False, jobs: int | None = None) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    newest_header = max(os.path.getmtime(h) for h in _headers())
    cmds, objs = [], []
    for src in _sources():
        obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), newest_header):
            cmds.append([nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj])
    procs = []
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for cmd, p in procs:
        out, _ = p.communicate()
        if verbose and out:
            print(out, end="")
        if p.returncode:
            failed.append((cmd[-3], out))
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(f"{src}:\n{out}" for src, out in failed))
    if cmds or force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-Xlinker", "--no-undefined"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
