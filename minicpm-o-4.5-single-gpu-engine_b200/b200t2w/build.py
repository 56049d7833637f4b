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
OPS_SRC = os.path.join(CSRC, "torch_ops.cpp")
OPS_PATH = os.path.join(LIB_DIR, "libt2w_torch_ops.so")

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
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-Xlinker", "--no-undefined",
               "-Xlinker", "-soname=libt2w_b200.so"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def build_ops(verbose: bool = False, force: bool = False) -> str:
    """The torch custom-op shim ``libt2w_torch_ops.so`` (``torch.ops.b200t2w.*``): ``csrc/torch_ops.cpp`` compiled with
    g++ against torch's headers and linked to ``libt2w_b200.so`` (found beside it through the rpath)."""
    import torch

    lib = build(verbose=verbose, force=force)
    deps = [OPS_SRC, lib] + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    if not force and os.path.exists(OPS_PATH) and os.path.getmtime(OPS_PATH) >= max(os.path.getmtime(d) for d in deps):
        return OPS_PATH
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    incs = [os.path.join(torch.__path__[0], "include"), os.path.join(torch.__path__[0], "include", "torch", "csrc", "api",
                                                                      "include"), os.path.join(cuda_home, "include"),
            INCLUDE]
    torch_lib = os.path.join(torch.__path__[0], "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = OPS_PATH + ".tmp"
    # the system g++ (a CXX wrapper may link libstdc++ statically: the shim must share torch's C++ runtime, or an
    # exception thrown by an op cannot unwind through torch's dispatcher)
    cxx = shutil.which("g++", path="/usr/bin:/bin") or "g++"
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{i}" for i in incs], OPS_SRC, "-o", tmp, f"-L{torch_lib}", f"-L{LIB_DIR}", "-lc10", "-lc10_cuda",
           "-ltorch_cpu", "-ltorch", "-l:libt2w_b200.so", "-Wl,--no-as-needed", "-lstdc++", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}",
           "-Wl,--no-undefined"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OPS_PATH)
    return OPS_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
    print(build_ops(verbose="-v" in sys.argv, force="-f" in sys.argv))
