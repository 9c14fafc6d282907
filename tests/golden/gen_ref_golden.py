"""Record the reference's own CUDA kernels' outputs as golden fixtures.

Runs on a machine with a GPU. It loads the reference kernels built from the reference
sources by ``oracle/build_ref.py`` (``oracle/_ref/fussim_ref_cuda.so``), feeds them
seeded CPU-generated inputs, and saves everything to one ``.pt`` file:

* FP32 path, ``fusedssim(ws, C1, C2, img1, img2, train=True)`` (``csrc/ssim.cu:603-619``):
  the SSIM map and the three partials; ``fusedssim_backward`` (``csrc/ssim.cu:621-640``)
  with ``dL_dmap`` = ones (same padding) and with the zero-padded valid-crop ones
  (the scatter of ``fussim/__init__.py:388-390``).
* FP16 path, ``fusedssim_fp16_train`` / ``fusedssim_fp16_backward``
  (``csrc/ssim_fp16.cu:807-842``) on the half-cast inputs, and the map-only
  ``fusedssim_fp16`` (``csrc/ssim_fp16.cu:791-805``).

The committed fixture ``ref_kernels.pt`` was produced with
``python tests/golden/gen_ref_golden.py --out <dir>`` on a B200 and copied here.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from fussim_b200 import synthetic  # noqa: E402
from oracle import build_ref  # noqa: E402

C1 = 0.01 ** 2
C2 = 0.03 ** 2

# (name, shape, seed): one case that reaches the reference's interior fast path
# (tiles whose halo lies fully inside the image), one thin odd-shaped case.
CASES = [("a", (1, 2, 40, 45), 1234), ("b", (2, 1, 37, 19), 99)]


def record(ext, shape, seed):
    img1, img2 = synthetic.pair_uniform(shape, seed)
    out = {"img1": img1.clone(), "img2": img2.clone()}
    d1, d2 = img1.cuda(), img2.cuda()
    for ws in (7, 9, 11):
        h = (ws - 1) // 2
        m, p0, p1, p2 = ext.fusedssim(ws, C1, C2, d1, d2, True)
        ones = torch.ones_like(m)
        g_same = ext.fusedssim_backward(ws, C1, C2, d1, d2, ones, p0, p1, p2)
        dl = torch.zeros_like(m)
        dl[:, :, h:-h, h:-h] = 1.0
        g_valid = ext.fusedssim_backward(ws, C1, C2, d1, d2, dl, p0, p1, p2)
        m_inf = ext.fusedssim(ws, C1, C2, d1, d2, False)[0]
        out[f"fp32_ws{ws}_map"] = m.cpu()
        out[f"fp32_ws{ws}_map_infer"] = m_inf.cpu()
        out[f"fp32_ws{ws}_grad_same"] = g_same.cpu()
        out[f"fp32_ws{ws}_grad_valid"] = g_valid.cpu()
        if ws == 11:
            out["fp32_ws11_dm_dmu1"] = p0.cpu()
            out["fp32_ws11_dm_dsigma1_sq"] = p1.cpu()
            out["fp32_ws11_dm_dsigma12"] = p2.cpu()

        h1, h2 = d1.half(), d2.half()
        hm, q0, q1, q2 = ext.fusedssim_fp16_train(ws, C1, C2, h1, h2)
        hg = ext.fusedssim_fp16_backward(ws, C1, C2, h1, h2, torch.ones_like(hm), q0, q1, q2)
        hm_inf = ext.fusedssim_fp16(ws, C1, C2, h1, h2)
        out[f"fp16_ws{ws}_map"] = hm.cpu()
        out[f"fp16_ws{ws}_map_infer"] = hm_inf.cpu()
        out[f"fp16_ws{ws}_grad_same"] = hg.cpu()
        if ws == 11:
            out["fp16_ws11_dm_dmu1"] = q0.cpu()
            out["fp16_ws11_dm_dsigma1_sq"] = q1.cpu()
            out["fp16_ws11_dm_dsigma12"] = q2.cpu()
    torch.cuda.synchronize()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(ROOT, "tests", "golden"))
    a = ap.parse_args()
    os.makedirs(a.out, exist_ok=True)
    ext = build_ref.load()
    fixture = {"C1": C1, "C2": C2, "cases": {}}
    for name, shape, seed in CASES:
        fixture["cases"][name] = {"shape": shape, "seed": seed, **record(ext, shape, seed)}
    path = os.path.join(a.out, "ref_kernels.pt")
    torch.save(fixture, path)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
