"""The fused 3DGS photometric loss (1 - l) * mean|x - y| + l * (1 - SSIM) against the oracle.

Reference usage: tests/test_amp.py:223-227 (fused_ssim plus a separate torch L1 term). The
fused form must give the same value and gradient as that composition; the ground truth
here is the float64 oracle (SSIM value and gradient by autograd over the conv2d SSIM with
the kernels' tables) plus the exact L1 term, on seeded inputs.
"""

import pytest
import torch

import fussim_b200 as fb
from fussim_b200 import synthetic
from oracle import ssim_oracle as O

pytestmark = pytest.mark.gpu


def _truth(a, b, lam, ws, padding):
    val, grad = O.loss_and_grad(a, b, ws, padding)  # SSIM mean and its gradient (float64)
    x = a.double()
    d = x - b.double()
    n = x.numel()
    value = (1 - lam) * d.abs().mean() + lam * (1 - val)
    g = (1 - lam) * torch.sign(d) / n - lam * grad
    return value.item(), g


@pytest.mark.parametrize("ws", [7, 9, 11])
@pytest.mark.parametrize("padding", ["same", "valid"])
@pytest.mark.parametrize("lam", [0.0, 0.2, 1.0])
def test_value_and_grad_fp32(ws, padding, lam):
    a, b = synthetic.pair_noise((2, 3, 70, 133), 0.1, seed=7 + ws)
    want_v, want_g = _truth(a, b, lam, ws, padding)
    x = a.cuda().requires_grad_(True)
    v = fb.l1_dssim_loss(x, b.cuda(), lambda_dssim=lam, padding=padding, window_size=ws)
    v.backward()
    assert v.dtype == torch.float32 and v.dim() == 0
    assert abs(v.item() - want_v) <= 1e-5
    g = x.grad.double().cpu()
    assert (g - want_g).abs().max().item() <= 1e-5 * want_g.abs().max().item() + 1e-12


def test_matches_unfused_composition_and_inference():
    a, b = synthetic.make_pair("unit_256")
    a, b = a.cuda(), b.cuda()
    lam = 0.2
    x1 = a.clone().requires_grad_(True)
    v1 = fb.l1_dssim_loss(x1, b, lambda_dssim=lam)
    v1.backward()
    x2 = a.clone().requires_grad_(True)
    v2 = (1 - lam) * (x2 - b).abs().mean() + lam * (1 - fb.fused_ssim(x2, b))
    v2.backward()
    assert abs(v1.item() - v2.item()) <= 1e-6
    assert (x1.grad - x2.grad).abs().max().item() <= 1e-6 * x2.grad.abs().max().item() + 1e-12
    with torch.no_grad():
        v3 = fb.l1_dssim_loss(a, b, lambda_dssim=lam)
    assert v3.item() == v1.item()


def test_equal_pixels_have_no_l1_gradient():
    a, b = synthetic.pair_noise((1, 3, 64, 96), 0.05, seed=3)
    b[:, :, 10:30, 20:60] = a[:, :, 10:30, 20:60]  # exact equality: sign(0) = 0
    want_v, want_g = _truth(a, b, 0.2, 11, "same")
    x = a.cuda().requires_grad_(True)
    v = fb.l1_dssim_loss(x, b.cuda())
    v.backward()
    assert abs(v.item() - want_v) <= 1e-5
    g = x.grad.double().cpu()
    assert (g - want_g).abs().max().item() <= 1e-5 * want_g.abs().max().item()


def test_deterministic():
    a, b = synthetic.make_pair("unit_256")
    outs = []
    for _ in range(2):
        x = a.cuda().requires_grad_(True)
        v = fb.l1_dssim_loss(x, b.cuda())
        v.backward()
        outs.append((v.item(), x.grad.clone()))
    assert outs[0][0] == outs[1][0]
    assert torch.equal(outs[0][1], outs[1][1])


def test_fp16_autocast():
    a, b = synthetic.pair_noise((2, 3, 96, 128), 0.1, seed=11)
    a, b = a.cuda(), b.cuda()
    lam = 0.2
    x1 = a.clone().requires_grad_(True)
    with torch.autocast("cuda"):
        v1 = fb.l1_dssim_loss(x1, b, lambda_dssim=lam)
    v1.backward()
    x2 = a.clone().requires_grad_(True)
    with torch.autocast("cuda"):
        s = fb.fused_ssim(x2, b)
    ah, bh = a.half().float(), b.half().float()  # the FP16 path sees half-rounded images
    l1 = (x2 + (ah - a).detach() - bh).abs().mean()
    v2 = (1 - lam) * l1 + lam * (1 - s)
    v2.backward()
    assert v1.dtype == torch.float32
    assert abs(v1.item() - v2.item()) <= 2e-3
    assert (x1.grad - x2.grad).abs().max().item() <= 2e-3 * x2.grad.abs().max().item()


def test_argument_errors():
    a = torch.rand(1, 3, 32, 32, device="cuda")
    with pytest.raises(ValueError, match="lambda_dssim"):
        fb.l1_dssim_loss(a, a, lambda_dssim=1.5)
    with pytest.raises(ValueError, match="padding"):
        fb.l1_dssim_loss(a, a, padding="reflect")
    with pytest.raises(ValueError, match="window_size"):
        fb.l1_dssim_loss(a, a, window_size=5)
