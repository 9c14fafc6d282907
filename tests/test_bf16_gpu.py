"""The native bfloat16 input path.

The reference has no bfloat16 kernel (its FP32 kernels reject bfloat16 tensors, and under
autocast every dtype goes to its FP16 kernels, which this engine keeps). Outside autocast a
bfloat16 pair is read natively here: the kernels widen each element to FP32 and run the
FP32 path's arithmetic with the FP32 taps, so the bfloat16 gradient must equal the FP32
gradient on the widened images rounded to bfloat16, bit for bit, and the value must agree
to 1e-7 (the deterministic reduction rounds once per column run, and the two kernels'
persistent grids, hence their run boundaries, may differ). Checked for both paddings,
windows 7/9/11, and the per-image wrapper.
"""

import pytest
import torch

import fussim_b200 as fb
from fussim_b200 import synthetic
from tests import refpath

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(2, 3, 64, 96), (1, 2, 37, 45), (1, 3, 1080, 1920)])
@pytest.mark.parametrize("ws", (7, 9, 11))
@pytest.mark.parametrize("padding", ["same", "valid"])
def test_bf16_matches_fp32_on_widened_inputs(device, shape, ws, padding):
    if shape[2] == 1080 and ws != 11:
        pytest.skip("the 1080p frame runs with the default window only")
    a, b = synthetic.pair_noise(shape, 0.1, seed=11000 + ws)
    a16, b16 = a.bfloat16().cuda(), b.bfloat16().cuda()
    v_b, g_b = refpath.value_and_grad(
        lambda x, y: fb.fused_ssim(x, y, padding=padding, window_size=ws), a16, b16)
    v_f, g_f = refpath.value_and_grad(
        lambda x, y: fb.fused_ssim(x, y, padding=padding, window_size=ws),
        a16.float(), b16.float())
    assert v_b.dtype == torch.float32 and g_b.dtype == torch.bfloat16
    assert abs(v_b.item() - v_f.item()) <= 1e-7
    assert torch.equal(g_b, g_f.to(torch.bfloat16))


def test_bf16_per_image_ssim(device):
    a, b = synthetic.pair_noise((3, 3, 50, 61), 0.1, seed=12000)
    a16, b16 = a.bfloat16().cuda(), b.bfloat16().cuda()
    v_b = fb.ssim(a16, b16, data_range=1.0, size_average=False)
    v_f = fb.ssim(a16.float(), b16.float(), data_range=1.0, size_average=False)
    assert v_b.shape == (3,) and (v_b - v_f).abs().max().item() <= 1e-7


def test_bf16_with_fp32_partner_is_widened(device):
    """A bfloat16 image paired with a float32 one goes through the float32 path."""
    a, b = synthetic.pair_noise((1, 3, 40, 48), 0.1, seed=12001)
    a16 = a.bfloat16().cuda()
    v_mixed = fb.fused_ssim(a16, b.cuda(), train=False)
    v_f = fb.fused_ssim(a16.float(), b.cuda(), train=False)
    assert torch.equal(v_mixed, v_f)
