"""Golden vectors from the reference's own Python test oracle.

Imports ``reference_ssim`` from the reference checkout's ``tests/test_ssim.py`` (lines
34-61: the pytorch-ssim conv2d formula, window 11, sigma 1.5, zero padding) and records
its value and autograd gradient on seeded float64 inputs. That test module starts with
``from fussim import fussim``, a name the reference package never exported; a stand-in
module satisfying that import is installed first so the oracle functions can be loaded
unchanged.

Run here (CPU only): ``python tests/golden/gen_test_oracle_golden.py [--reference DIR]``.
Writes ``tests/golden/ref_test_oracle.pt``.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
CASES = [((1, 3, 32, 32), 7), ((2, 1, 23, 37), 8), ((1, 2, 48, 53), 9)]


def load_reference_test_module(reference: str):
    stub = types.ModuleType("fussim")
    stub.fussim = None
    sys.modules.setdefault("fussim", stub)
    path = os.path.join(reference, "tests", "test_ssim.py")
    spec = importlib.util.spec_from_file_location("reference_test_ssim", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None,
                    help="reference checkout (default: $FUSSIM_REFERENCE_DIR or the container's)")
    ap.add_argument("--out", default=os.path.join(HERE, "ref_test_oracle.pt"))
    a = ap.parse_args()
    from oracle import build_ref

    mod = load_reference_test_module(a.reference or build_ref.reference_dir())
    out = {"source": "tests/test_ssim.py:reference_ssim", "cases": []}
    for shape, seed in CASES:
        g = torch.Generator().manual_seed(seed)
        img1 = torch.rand(shape, generator=g, dtype=torch.float64)
        img2 = (img1 + 0.1 * torch.randn(shape, generator=g, dtype=torch.float64)).clamp(0, 1)
        x = img1.clone().requires_grad_(True)
        val = mod.reference_ssim(x, img2, window_size=11)
        val.backward()
        out["cases"].append({"shape": shape, "seed": seed, "img1": img1, "img2": img2,
                             "value": val.detach(), "grad": x.grad.detach()})
    torch.save(out, a.out)
    print("wrote", a.out, os.path.getsize(a.out), "bytes")


if __name__ == "__main__":
    main()
