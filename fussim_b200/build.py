"""In-tree build of the engine for sm_100a.

Produces, next to this file:

* ``libfussim_b200.so``  the C-ABI library (nvcc, no torch), declared in
  ``include/fussim_b200.h``;
* ``_C.so``              the thin torch extension over that library (g++ against torch's
  headers, rpath ``$ORIGIN`` so it finds the library beside it).

Run ``python -m fussim_b200.build`` (or ``__graft_entry__.build()``). Nothing is cached
outside the repository, so the built files travel with a copy of the tree.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libfussim_b200.so")
EXT = os.path.join(PKG, "_C.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(home, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} (exit {res.returncode})")
    return res


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def engine_sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh"))]


def build_engine(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    deps = engine_sources() + [os.path.join(INCLUDE, "fussim_b200.h")]
    if not force and not _stale(LIB, deps):
        return LIB
    cus = [s for s in engine_sources() if s.endswith(".cu")]
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-shared", "-I", INCLUDE, "-o", LIB, *cus]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    res = _run(cmd, verbose)
    if ptxas_info:
        sys.stdout.write(res.stderr)
    return LIB


def build_torch_ext(force: bool = False, verbose: bool = False) -> str:
    # The extension links the library by name and finds it at run time, so a rebuilt
    # library does not require relinking the extension.
    deps = [os.path.join(CSRC, "torch_ext.cpp"), os.path.join(INCLUDE, "fussim_b200.h")]
    if not force and not _stale(EXT, deps):
        return EXT
    import torch
    from torch.utils import cpp_extension as ce

    incs = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], INCLUDE]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{i}" for i in incs], os.path.join(CSRC, "torch_ext.cpp"), "-o", EXT,
           *[f"-L{d}" for d in libdirs], f"-L{PKG}", "-lfussim_b200", "-lc10", "-ltorch",
           "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda", "-lcudart",
           "-Wl,-rpath,$ORIGIN"]
    _run(cmd, verbose)
    return EXT


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_engine(force=force, verbose=verbose)
    build_torch_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose=True)
    print(LIB)
    print(EXT)
