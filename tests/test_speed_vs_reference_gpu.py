"""The engine's fwd+bwd step against the reference's own CUDA kernels, on the same GPU.

The reference kernels are the reference's sources compiled for sm_100 with the reference's
own flags (oracle/build_ref.py); its step is the reference's Python sequence around them
(tests/refpath.py): fusedssim -> mean -> fusedssim_backward. Both steps run on the same
1x3x1080x1920 FP32 blob pair (the 3DGS training-step shape), with CUDA events around 50
back-to-back steps after a warm-up. The test asserts the engine's step is faster and prints
both times (run pytest with -s to see them).
"""

import pytest
import torch

import fussim_b200 as fb
from fussim_b200 import synthetic
from tests import refpath

pytestmark = pytest.mark.gpu


def _time_ms(fn, iters=50, warm=10):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    torch.cuda._sleep(20_000_000)  # ~10 ms: the host queues the steps before timing starts
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


@pytest.mark.parametrize("padding", ["same", "valid"])
def test_engine_step_is_faster_than_reference_kernels(ref_ext, padding):
    a, b = synthetic.make_pair("rgb_1080p", seed=102)
    x = a.cuda().requires_grad_(True)
    y = b.cuda()

    def ours():
        v = fb.fused_ssim(x, y, padding=padding)
        v.backward()
        x.grad = None

    def ref():
        v = refpath.reference_loss(ref_ext, x, y, 11, padding)
        v.backward()
        x.grad = None

    t_ref = _time_ms(ref)
    t_ours = _time_ms(ours)
    n = x.numel()
    print(f"\n1x3x1080x1920 fp32 {padding} fwd+bwd: reference kernels {t_ref * 1e3:.1f} us "
          f"({n / t_ref / 1e3:.0f} Mpix/s), engine {t_ours * 1e3:.1f} us "
          f"({n / t_ours / 1e3:.0f} Mpix/s), {t_ref / t_ours:.2f}x")
    assert t_ours < t_ref
