"""The fused loss path's two kernel families compute the same per-pixel results.

The column-streaming kernels (the default: one output column per thread, the vertical
window carried in registers) and the 4-row tile kernels (shared with the map entry points)
run the same arithmetic in the same order, so their partials and gradients must be bitwise
identical; the reduced values may differ only by the FP32 grouping of the per-thread sums
(|diff| <= 1e-7 here). The tile kernels are themselves pinned to the reference kernels by
test_parity_gpu.py; this file pins the streaming kernels to them on every path the fused
loss has: both paddings, windows 7/9/11, the clamp and per-image reductions, FP16 autocast,
bfloat16 images, the fused L1 term, shapes with partial strips and steps, images shorter
than one step, and a batch whose CTAs split column runs.
"""

import pytest
import torch

import fussim_b200 as fb
from fussim_b200 import synthetic
from fussim_b200.functional import _ensure_cuda_extension
from tests import refpath

pytestmark = pytest.mark.gpu

STREAM, TILE, AUTO = 0, 1, 2
SHAPES = [(1, 2, 40, 45), (2, 1, 37, 19), (1, 3, 64, 67), (2, 3, 96, 256), (1, 1, 5, 7),
          (2, 3, 37, 64), (1, 1, 5, 8), (1, 2, 130, 200), (3, 3, 200, 130)]


@pytest.fixture
def ext(device):
    e = _ensure_cuda_extension()
    yield e
    e.set_loss_kernels(AUTO)


def _both(ext, fn, a, b):
    out = []
    for fam in (STREAM, TILE):
        ext.set_loss_kernels(fam)
        out.append(refpath.value_and_grad(fn, a, b))
    ext.set_loss_kernels(AUTO)
    return out


def _check(res):
    (v_s, g_s), (v_t, g_t) = res
    # an empty valid crop gives NaN means on both sides
    assert torch.equal(torch.isnan(v_s), torch.isnan(v_t))
    ok = ~torch.isnan(v_t)
    assert (v_s[ok].double() - v_t[ok].double()).abs().max().item() <= 1e-7 if ok.any() else True
    assert torch.equal(g_s, g_t), (g_s.double() - g_t.double()).abs().max().item()


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("ws", (7, 9, 11))
@pytest.mark.parametrize("padding", ["same", "valid"])
def test_stream_matches_tile_fp32(ext, shape, ws, padding):
    a, b = synthetic.pair_noise(shape, 0.1, seed=13000 + ws)
    _check(_both(ext, lambda x, y: fb.fused_ssim(x, y, padding=padding, window_size=ws),
                 a.cuda(), b.cuda()))


@pytest.mark.parametrize("shape", SHAPES[:6])
@pytest.mark.parametrize("ws", (7, 11))
def test_stream_matches_tile_autocast(ext, shape, ws):
    a, b = synthetic.pair_noise(shape, 0.1, seed=14000 + ws)

    def f(x, y):
        with torch.autocast("cuda"):
            return fb.fused_ssim(x, y, window_size=ws)

    _check(_both(ext, f, a.cuda(), b.cuda()))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_stream_matches_tile_2byte_images(ext, dtype):
    a, b = synthetic.pair_noise((2, 3, 96, 136), 0.1, seed=15000)
    _check(_both(ext, lambda x, y: fb.fused_ssim(x, y), a.to(dtype).cuda(), b.to(dtype).cuda()))


@pytest.mark.parametrize("size_average", [True, False])
@pytest.mark.parametrize("nonneg", [False, True])
def test_stream_matches_tile_ssim_wrapper(ext, size_average, nonneg):
    a, b = synthetic.pair_noise((3, 2, 50, 61), 0.1, seed=16000)
    b = 1.0 - b if nonneg else b
    _check(_both(ext, lambda x, y: fb.ssim(x, y, data_range=1.0, size_average=size_average,
                                          nonnegative_ssim=nonneg), a.cuda(), b.cuda()))


@pytest.mark.parametrize("lam", [0.0, 0.2, 1.0])
def test_stream_matches_tile_l1_dssim(ext, lam):
    a, b = synthetic.pair_noise((2, 3, 70, 130), 0.1, seed=17000)
    _check(_both(ext, lambda x, y: fb.l1_dssim_loss(x, y, lambda_dssim=lam), a.cuda(),
                 b.cuda()))


def test_stream_matches_tile_partials_1080p(ext):
    """The forward's partials themselves, on the 1080p blob pair (bitwise)."""
    a, b = synthetic.make_pair("rgb_1080p", seed=102)
    a, b = a.cuda(), b.cuda()
    n = a.numel()
    outs = []
    for fam in (STREAM, TILE):
        ext.set_loss_kernels(fam)
        out, partials, sums = ext.loss_forward(a, b, 11, 0.01**2, 0.03**2, False, False, True, 1,
                                               False, 1.0 / n)
        outs.append((out, partials, sums))
    ext.set_loss_kernels(AUTO)
    assert torch.equal(outs[0][1], outs[1][1])
    assert abs(outs[0][0].item() - outs[1][0].item()) <= 1e-7


def test_stream_matches_tile_whole_batch(ext):
    """A batch of 4 1024^2 planes: the grid splits column runs between CTAs."""
    a, b = synthetic.pair_noise((4, 1, 1024, 1024), 0.1, seed=18000)
    _check(_both(ext, lambda x, y: fb.fused_ssim(x, y), a.cuda(), b.cuda()))


def test_set_loss_kernels_rejects_unknown_family(ext):
    with pytest.raises(RuntimeError, match="family"):
        ext.set_loss_kernels(7)
