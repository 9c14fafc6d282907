"""The CPU oracle, pinned against the reference's own outputs (runs without a GPU).

* ``ref_test_oracle.pt``: the reference's test oracle ``reference_ssim`` (tests/test_ssim.py,
  window 11) — value within 1e-8, gradient within 1e-6 of its max (the oracle uses the
  kernels' float32 tables in float64; the test oracle builds its window in float32).
* ``ref_kernels.pt``: the reference CUDA kernels on a B200, windows 7/9/11, FP32 and FP16 —
  maps within 1e-5, gradients (dL/dmap = 1) within 1e-5 * max|g| + 1e-5.
"""

import os

import numpy as np
import pytest
import torch

from oracle import ssim_oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def test_oracle_golden():
    return torch.load(os.path.join(GOLDEN, "ref_test_oracle.pt"))


@pytest.fixture(scope="module")
def kernel_golden():
    return torch.load(os.path.join(GOLDEN, "ref_kernels.pt"))


def test_matches_reference_test_oracle(test_oracle_golden):
    assert test_oracle_golden["source"].startswith("tests/test_ssim.py")
    for c in test_oracle_golden["cases"]:
        v, g = O.loss_and_grad(c["img1"], c["img2"], 11, "same")
        assert abs(v.item() - c["value"].item()) < 1e-8
        assert (g - c["grad"]).abs().max().item() <= 1e-6 * c["grad"].abs().max().item()


@pytest.mark.parametrize("name", ["a", "b"])
@pytest.mark.parametrize("ws", [7, 9, 11])
@pytest.mark.parametrize("half", [False, True])
def test_matches_reference_kernels(kernel_golden, name, ws, half):
    case = kernel_golden["cases"][name]
    tag = "fp16" if half else "fp32"
    m, p0, p1, p2 = O.ssim_map_and_partials(case["img1"], case["img2"], ws, half=half)
    assert (m - case[f"{tag}_ws{ws}_map"].double()).abs().max().item() <= 1e-5
    assert (m - case[f"{tag}_ws{ws}_map_infer"].double()).abs().max().item() <= 1e-5
    g = O.backward_closed_form(case["img1"], case["img2"], torch.ones_like(m), (p0, p1, p2), ws,
                               half=half)
    ref = case[f"{tag}_ws{ws}_grad_same"].double()
    assert (g - ref).abs().max().item() <= 1e-5 + 1e-5 * ref.abs().max().item()
    if not half:
        dl = torch.zeros_like(m)
        dl[:, :, ws // 2:-(ws // 2), ws // 2:-(ws // 2)] = 1.0
        gv = O.backward_closed_form(case["img1"], case["img2"], dl, (p0, p1, p2), ws)
        refv = case[f"fp32_ws{ws}_grad_valid"].double()
        assert (gv - refv).abs().max().item() <= 1e-5 + 1e-5 * refv.abs().max().item()
    if ws == 11:
        for k, nm in enumerate(("dm_dmu1", "dm_dsigma1_sq", "dm_dsigma12")):
            ours = (p0, p1, p2)[k]
            r = case[f"{tag}_ws11_{nm}"].double()
            assert (ours - r).abs().max().item() <= 1e-5 + 1e-5 * r.abs().max().item()


@pytest.mark.parametrize("ws", [7, 9, 11])
def test_closed_form_chain_equals_autograd(ws):
    g = torch.Generator().manual_seed(ws)
    a = torch.rand(2, 2, 19, 23, generator=g, dtype=torch.float64)
    b = (a + 0.2 * torch.randn(a.shape, generator=g, dtype=torch.float64)).clamp(0, 1)
    m, p0, p1, p2 = O.ssim_map_and_partials(a, b, ws)
    gc = O.backward_closed_form(a, b, torch.ones_like(m), (p0, p1, p2), ws)
    _, ga = O.loss_and_grad(a, b, ws, "same")
    assert (ga * m.numel() - gc).abs().max().item() < 1e-10


def test_known_answers():
    g = torch.Generator().manual_seed(3)
    x = torch.rand(1, 3, 32, 32, generator=g, dtype=torch.float64)
    for ws in (7, 9, 11):
        # identical images -> 1 (reference tests/test_window_sizes.py:31-34)
        assert abs(O.loss_and_grad(x, x, ws)[0].item() - 1.0) < 1e-5
        # constant 0.5 -> 1 (tests/test_window_sizes.py:124-129)
        c = torch.full((1, 3, 32, 32), 0.5, dtype=torch.float64)
        assert abs(O.loss_and_grad(c, c, ws)[0].item() - 1.0) < 1e-5
    # zeros vs ones -> low SSIM (tests/test_equivalence.py:329-336)
    z, o = torch.zeros(1, 3, 32, 32), torch.ones(1, 3, 32, 32)
    assert O.loss_and_grad(z, o, 11)[0].item() < 0.5


def test_weight_tables_match_kernel_source():
    """The FP32 and half-rounded tap tables in the CUDA source equal the oracle's."""
    import re

    src = open(os.path.join(os.path.dirname(__file__), "..", "fussim_b200", "csrc",
                            "ssim_kernels.cuh")).read()
    body = src[src.index("c_taps[2][3][11] = {"):]
    body = body[:body.index("};")]
    vals = [float.fromhex(v[:-1]) if v.startswith("0x") else float(v[:-1])
            for v in re.findall(r"(0x[0-9a-fp.+-]+f|[0-9.]+(?:e-?\d+)?f)", body)]
    assert len(vals) == 66
    tables = np.asarray(vals, dtype=np.float32).reshape(2, 3, 11)
    for hi, half in enumerate((False, True)):
        for wi, ws in enumerate((7, 9, 11)):
            np.testing.assert_array_equal(tables[hi, wi, :ws], O.taps(ws, half).astype(np.float32))
    # the 9-tap table sums to 0.54 and the 7-tap one is a sigma=1 kernel (not sigma=1.5)
    assert abs(O.taps(9).sum() - 0.54) < 1e-6
    assert abs(O.taps(7).sum() - 1.0) < 1e-6
