"""Build the reference's own CUDA kernels as a torch extension, for parity checks only.

TEST INFRASTRUCTURE. This compiles the unmodified reference sources
(`csrc/ssim.cu`, `csrc/ssim_fp16.cu`, `csrc/ext.cpp` of OpsiClear/fussim) from where
they lie in the read-only reference checkout, with the reference's own nvcc flags
(`setup.py:157` for C++, `setup.py:323-328` for nvcc: `-O3 --maxrregcount=32
--use_fast_math -std=c++17`) and the B200 arch the reference ships for
(`setup.py:304`: `compute_100`/`sm_100`). Output goes to `oracle/_ref/` only, which is
git-ignored. Nothing in the product imports it: the tests, `smoke()` and the reference
timing test load it as the checker / the competitor.

The module exposes the five reference entry points (`csrc/ext.cpp:11-17`):
`fusedssim`, `fusedssim_backward`, `fusedssim_fp16`, `fusedssim_fp16_train`,
`fusedssim_fp16_backward`.

Usage: python oracle/build_ref.py [--reference DIR]
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
MODULE_NAME = "fussim_ref_cuda"


def reference_dir() -> str:
    """Where the read-only reference checkout lies: $FUSSIM_REFERENCE_DIR, else the build
    container's checkout location. Only the build recipes read it; nothing does at run time."""
    return os.environ.get("FUSSIM_REFERENCE_DIR", "/root/reference")


def built_path() -> str | None:
    """Path of the built reference extension, or None if it has not been built."""
    hits = sorted(glob.glob(os.path.join(REF_DIR, MODULE_NAME + "*.so")))
    return hits[0] if hits else None


def build(reference: str | None = None, verbose: bool = False) -> str:
    reference = reference or reference_dir()
    csrc = os.path.join(reference, "csrc")
    sources = [os.path.join(csrc, f) for f in ("ssim.cu", "ssim_fp16.cu", "ext.cpp")]
    for s in sources:
        if not os.path.isfile(s):
            raise FileNotFoundError(f"reference source missing: {s}")
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils import cpp_extension

    build_dir = os.path.join(REF_DIR, "build")
    os.makedirs(build_dir, exist_ok=True)
    cpp_extension.load(
        name=MODULE_NAME,
        sources=sources,
        extra_include_paths=[csrc],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=[
            "-O3",
            "--maxrregcount=32",
            "--use_fast_math",
            "-std=c++17",
            "-gencode=arch=compute_100,code=sm_100",
        ],
        build_directory=build_dir,
        verbose=verbose,
        is_python_module=True,
        with_cuda=True,
    )
    so = os.path.join(build_dir, MODULE_NAME + ".so")
    dst = os.path.join(REF_DIR, MODULE_NAME + ".so")
    shutil.copy2(so, dst)
    return dst


def load():
    """Import the prebuilt reference extension from oracle/_ref (no rebuild)."""
    import importlib.machinery
    import importlib.util

    path = built_path()
    if path is None:
        raise ImportError("reference kernels not built: run python oracle/build_ref.py")
    import torch  # noqa: F401  (the extension links against libtorch)

    loader = importlib.machinery.ExtensionFileLoader(MODULE_NAME, path)
    spec = importlib.util.spec_from_file_location(MODULE_NAME, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="reference checkout "
                    "(default: $FUSSIM_REFERENCE_DIR or the container's checkout)")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    out = build(a.reference, a.verbose)
    print(out)
    sys.exit(0)
