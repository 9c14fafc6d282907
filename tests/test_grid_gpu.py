"""Results do not depend on the size of the persistent grids.

`fssim_set_reserved_sms(n)` shrinks every persistent grid to the SMs left over, which moves
the boundaries of the CTAs' row ranges (and, at one SM, gives each CTA many strips and
images). Every per-pixel value is computed from the same taps in the same order whoever
owns the pixel, and the row steps stay aligned to the image, so maps and gradients must be
bit-identical for every grid. The reduced values add one 2^-28 fixed-point rounding per
column run, and the runs move with the grid: they may differ by those roundings only
(|diff| <= 1e-6, far below any FP32 parity bound).
"""

import pytest
import torch

import fussim_b200 as fb
from fussim_b200 import synthetic
from fussim_b200.functional import _ensure_cuda_extension

pytestmark = pytest.mark.gpu


def _run(a, b):
    x = a.clone().requires_grad_(True)
    v = fb.fused_ssim(x, b)
    v.backward()
    x2 = a.clone().requires_grad_(True)
    l = fb.l1_dssim_loss(x2, b, lambda_dssim=0.2, padding="valid")
    l.backward()
    with torch.no_grad():
        per = fb.ssim(a, b, size_average=False, nonnegative_ssim=True)
    with torch.autocast("cuda"):
        x3 = a.clone().requires_grad_(True)
        h = fb.fused_ssim(x3, b)
    h.backward()
    values = [v.detach(), l.detach(), per, h.detach()]
    return values, [x.grad, x2.grad, x3.grad]


@pytest.mark.parametrize("shape", [(3, 3, 150, 230), (1, 1, 1080, 64), (5, 2, 37, 19)])
def test_bit_identical_across_grid_sizes(shape):
    ext = _ensure_cuda_extension()
    a, b = synthetic.pair_noise(shape, 0.1, seed=sum(shape))
    a, b = a.cuda(), b.cuda()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    try:
        ext.set_reserved_sms(0)
        want = _run(a, b)
        for n in (1, sms // 2, sms - 1, sms + 10):
            ext.set_reserved_sms(n)
            got = _run(a, b)
            torch.cuda.synchronize()
            for i, (g, w) in enumerate(zip(got[0], want[0])):
                d = (g.double() - w.double()).abs().max().item()
                assert d <= 1e-6, f"value {i} differs by {d} with {n} SMs reserved"
            for i, (g, w) in enumerate(zip(got[1], want[1])):
                assert torch.equal(g, w), f"gradient {i} differs with {n} SMs reserved"
    finally:
        ext.set_reserved_sms(0)
