"""Failure paths of the kernels' bounded waits, made to run out on purpose, on one GPU.

Nothing here faults, traps or hangs the GPU. Each wait has a limit after which the kernel
records a bit in the device error flag and returns:

* staging: with the staging wait limit set to 0 polls, every step staged by the tensor
  memory accelerator gives up at once (after its copies in flight have landed). A forward
  with a reduction must still complete its reduction: NaN outputs, error bit 0, and a
  workspace left zeroed, so the next call on the same stream (same cached workspace)
  returns the correct value. The backward records bit 0 as well.
* sharded gather: one rank's gather over a world of 2 whose second slot nobody publishes
  (both mailbox entries point at this rank's own mailbox) must give up after its timeout
  with NaN and error bit 1.
"""

import math

import pytest
import torch

import fussim_b200 as fb
from fussim_b200 import synthetic
from fussim_b200.functional import _ensure_cuda_extension

pytestmark = pytest.mark.gpu

SHAPE = (2, 3, 64, 96)  # W * 4 bytes is a multiple of 16: staged with TMA boxes


@pytest.fixture
def ext(device):
    e = _ensure_cuda_extension()
    fb.poll_device_error(clear=True)
    yield e
    e.set_staging_wait_limit(-1)
    e.set_gather_timeout_us(0)
    fb.poll_device_error(clear=True)


def test_staging_timeout_gives_nan_and_leaves_workspace_clean(ext):
    a, b = synthetic.pair_noise(SHAPE, 0.1, seed=3)
    a, b = a.cuda(), b.cuda()
    x = a.clone().requires_grad_(True)
    want = fb.fused_ssim(x, b).item()
    want_img = fb.ssim(a, b, data_range=1.0, size_average=False)
    assert fb.poll_device_error() == 0

    ext.set_staging_wait_limit(0)
    v = fb.fused_ssim(x, b)                                  # scalar reduction
    per = fb.ssim(a, b, data_range=1.0, size_average=False)  # per-image reduction
    torch.cuda.synchronize()
    ext.set_staging_wait_limit(-1)
    assert math.isnan(v.item())
    assert torch.isnan(per).all() and per.shape == (SHAPE[0],)
    code = fb.poll_device_error(clear=False)
    assert code & 1, f"device error flag {code:#x}"
    with pytest.raises(RuntimeError, match="staging"):
        fb.check_device_errors()
    assert fb.poll_device_error() == 0  # check_device_errors cleared it

    # the same stream's cached workspace is clean again: exact results on the next calls
    assert fb.fused_ssim(x, b).item() == want
    assert torch.equal(fb.ssim(a, b, data_range=1.0, size_average=False), want_img)
    assert fb.poll_device_error() == 0


def test_backward_staging_timeout_sets_flag(ext):
    a, b = synthetic.pair_noise(SHAPE, 0.1, seed=4)
    x = a.cuda().requires_grad_(True)
    v = fb.fused_ssim(x, b.cuda())
    torch.cuda.synchronize()
    ext.set_staging_wait_limit(0)
    v.backward()
    torch.cuda.synchronize()
    ext.set_staging_wait_limit(-1)
    assert fb.poll_device_error() & 1


def test_gather_timeout_gives_nan_and_sets_flag(ext):
    mb = ext.dp_mailbox_alloc(2)
    try:
        ext.set_gather_timeout_us(20_000)  # 20 ms
        out = torch.zeros((), device="cuda")
        # world of 2 on one GPU: slot 1 is never published for seq 5
        ext.dp_gather(out, 1.0, 2, 0, 5, [mb, mb])
        torch.cuda.synchronize()
        assert math.isnan(out.item())
        assert fb.poll_device_error() & 2
    finally:
        ext.dp_mailbox_free(mb)


def test_single_rank_exchange_round_trip(ext):
    """World of 1 through the mailbox path: the gathered value equals the local loss."""
    a, b = synthetic.pair_noise(SHAPE, 0.1, seed=5)
    a, b = a.cuda(), b.cuda()
    mb = ext.dp_mailbox_alloc(1)
    try:
        n = a.numel()
        out, _ = ext.loss_forward_dp(a, b, 11, 0.01**2, 0.03**2, False, False, 1.0 / n, 1, 0, 1,
                                     [mb])
        ext.dp_gather(out, 1.0 / n, 1, 0, 1, [mb])
        torch.cuda.synchronize()
        assert abs(out.item() - fb.fused_ssim(a, b, train=False).item()) <= 1e-7
        assert fb.poll_device_error() == 0
    finally:
        ext.dp_mailbox_free(mb)
