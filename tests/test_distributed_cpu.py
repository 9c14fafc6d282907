"""The batch-sharded path (fussim_b200.distributed) on 2 gloo ranks, on the CPU.

The CUDA kernels cannot run without a GPU, so in these child processes each rank's local
forward and backward are replaced by the float64 oracle; the oracle is only the stand-in
for the kernel here. What is under test is the host logic of the sharded path: the global
pixel count (one all-reduce of the shard counts), the 1/N_global scale, the async
all-reduce of the scalar, and the local backward with the global scale. The value on every
rank must equal the mean SSIM of the concatenated global batch, and each rank's gradient the
matching slice of the global gradient (padding same and valid, uneven shards).
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fussim_b200 import synthetic
from oracle import ssim_oracle as O

WORLD = 2
SHARDS = (1, 2)              # images per rank (uneven on purpose)
SHAPE = (3, 24, 37)          # C, H, W


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _crop_mask(shape, window_size, valid):
    mask = torch.ones(shape, dtype=torch.float64)
    if valid:
        h = (window_size - 1) // 2
        mask.zero_()
        mask[:, :, h:shape[2] - h, h:shape[3] - h] = 1.0
    return mask


def _oracle_local_forward(a, b, window_size, C1, C2, valid, train, scale, clamp=False,
                          per_image=False):
    """Stand-in for the fused forward kernel: (local sum * scale, or the per-image sums *
    scale; partials masked by the crop and, with clamp, by map > 0)."""
    m, p0, p1, p2 = O.ssim_map_and_partials(a, b, window_size, C1, C2)
    mask = _crop_mask(a.shape, window_size, valid)
    if clamp:
        mask = mask * (m > 0)
    if per_image:
        out = ((m * mask).sum(dim=(1, 2, 3)) * scale).to(torch.float32)
    else:
        out = torch.tensor([float((m * mask).sum()) * scale], dtype=torch.float32)
    partials = torch.stack([p0 * mask, p1 * mask, p2 * mask]).to(torch.float32)
    return out, partials


def _oracle_local_backward(grad_out, a, b, partials, window_size, scale, grad_dtype,
                           per_image=False):
    """Stand-in for the fused backward kernel: dL/dimg1 with dL/dmap = grad_out * scale
    (per image with ``per_image``)."""
    if per_image:
        dl = (grad_out.double() * scale).view(-1, 1, 1, 1).expand(a.shape).contiguous()
    else:
        dl = torch.full(a.shape, float(grad_out) * scale, dtype=torch.float64)
    g = O.backward_closed_form(a, b, dl, tuple(partials.to(torch.float64)), window_size)
    return g.to(torch.float32)


MSSSIM_CASES = [(True, False), (False, False), (True, True), (False, True)]
IMAGE_WEIGHTS = (1.0, -2.0, 0.5)    # loss = sum_i w_i * ssim_i over the global batch


def _msssim_pair():
    a, b = _global_pair()
    return a, (1.0 - b) * 0.5 + 0.5 * a   # partly anti-correlated: some map values < 0


def _msssim_reference(size_average, nonneg):
    """float64 value and dLoss/dX of the pytorch-msssim form over the global batch."""
    a, b = _msssim_pair()
    C1, C2 = 0.01**2, 0.03**2
    m, p0, p1, p2 = O.ssim_map_and_partials(a, b, 11, C1, C2)
    mask = _crop_mask(a.shape, 11, True)
    if nonneg:
        mask = mask * (m > 0)
    n_img = SHAPE[0] * (SHAPE[1] - 10) * (SHAPE[2] - 10)    # valid-crop pixels per image
    w = torch.tensor(IMAGE_WEIGHTS, dtype=torch.float64)
    if size_average:
        val = (m * mask).sum() / (a.shape[0] * n_img)
        dl = mask / (a.shape[0] * n_img)
    else:
        val = (m * mask).sum(dim=(1, 2, 3)) / n_img
        dl = mask * (w / n_img).view(-1, 1, 1, 1)
    g = O.backward_closed_form(a, b, dl, (p0 * mask, p1 * mask, p2 * mask), 11)
    return val, g


def _global_pair():
    return synthetic.pair_noise((sum(SHARDS),) + SHAPE, 0.1, seed=23)


def _worker(rank, port, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from fussim_b200 import distributed as D

        D._local_forward = _oracle_local_forward
        D._local_backward = _oracle_local_backward
        a_all, b_all = _global_pair()
        lo = sum(SHARDS[:rank])
        results = {}
        for padding in ("same", "valid"):
            for async_op in (True, False):
                a = a_all[lo:lo + SHARDS[rank]].clone().requires_grad_(True)
                b = b_all[lo:lo + SHARDS[rank]].clone()
                if async_op:
                    v, work = D.fused_ssim_dp(a, b, padding=padding, async_op=True)
                    v.backward()   # the local backward runs while the all-reduce is in flight
                    work.wait()
                else:
                    v = D.fused_ssim_dp(a, b, padding=padding)
                    v.backward()
                # plain numpy across the process boundary (no shared-memory tensor handles)
                results[(padding, async_op)] = (float(v.detach()), a.grad.numpy().copy())
        a_all, b_all = _msssim_pair()
        for size_average, nonneg in MSSSIM_CASES:
            a = a_all[lo:lo + SHARDS[rank]].clone().requires_grad_(True)
            b = b_all[lo:lo + SHARDS[rank]].clone()
            v = D.ssim_dp(a, b, data_range=1.0, size_average=size_average,
                          nonnegative_ssim=nonneg)
            loss = v if size_average else (v * torch.tensor(IMAGE_WEIGHTS)).sum()
            loss.backward()
            with torch.no_grad():
                v_ng = D.ssim_dp(a, b, data_range=1.0, size_average=size_average,
                                 nonnegative_ssim=nonneg)
            results[("msssim", size_average, nonneg)] = (
                v.detach().numpy().copy(), v_ng.numpy().copy(), a.grad.numpy().copy())
        queue.put((rank, results))
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def rank_results():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = mp.start_processes(_worker, args=(_free_port(), queue), nprocs=WORLD, join=False,
                               start_method="spawn")
    # drain the queue before joining: a child cannot exit until its result has been read
    out = {}
    for _ in range(WORLD):
        rank, res = queue.get(timeout=180)  # a rank that failed raises in join below
        out[rank] = res
    while not procs.join(timeout=120):
        pass
    return out


@pytest.mark.parametrize("padding", ["same", "valid"])
@pytest.mark.parametrize("async_op", [True, False])
def test_sharded_value_and_grad_match_global_batch(rank_results, padding, async_op):
    a_all, b_all = _global_pair()
    val, grad = O.loss_and_grad(a_all, b_all, 11, padding)
    for rank in range(WORLD):
        v, g = rank_results[rank][(padding, async_op)]
        g = torch.from_numpy(g)
        assert abs(v - float(val)) <= 1e-6
        lo = sum(SHARDS[:rank])
        ref = grad[lo:lo + SHARDS[rank]]
        err = (g.double() - ref).abs().max().item()
        assert err <= 1e-5 * max(1e-12, ref.abs().max().item()) + 1e-12


@pytest.mark.parametrize("size_average,nonneg", MSSSIM_CASES)
def test_sharded_msssim_matches_global_batch(rank_results, size_average, nonneg):
    """ssim_dp: the global mean, or the whole batch's per-image vector on every rank, and
    each rank's gradient the slice of the global batch's (per-image weights included)."""
    val, grad = _msssim_reference(size_average, nonneg)
    val = val.reshape(-1).to(torch.float64)
    for rank in range(WORLD):
        v, v_ng, g = rank_results[rank][("msssim", size_average, nonneg)]
        for got in (v, v_ng):
            got = torch.from_numpy(got).reshape(-1).double()
            assert got.shape == val.shape
            assert (got - val).abs().max().item() <= 1e-6
        lo = sum(SHARDS[:rank])
        ref = grad[lo:lo + SHARDS[rank]]
        err = (torch.from_numpy(g).double() - ref).abs().max().item()
        assert err <= 1e-5 * max(1e-12, ref.abs().max().item()) + 1e-12


def test_msssim_reference_exercises_the_clamp():
    a, b = _msssim_pair()
    m = O.ssim_map_and_partials(a, b, 11, 0.01**2, 0.03**2)[0]
    h = 5
    inner = m[:, :, h:-h, h:-h]
    assert (inner < 0).any() and (inner > 0).any()


def test_sharded_argument_errors():
    from fussim_b200 import distributed as D

    a = torch.rand(1, 3, 16, 16)
    with pytest.raises(ValueError, match="padding"):
        D.fused_ssim_dp(a, a, padding="reflect")
    with pytest.raises(ValueError, match="window_size"):
        D.fused_ssim_dp(a, a, window_size=5)
    with pytest.raises(ValueError, match="win_size"):
        D.ssim_dp(a, a, win_size=5)
    with pytest.raises(ValueError, match="win_sigma"):
        D.ssim_dp(a, a, win_sigma=2.0)
    with pytest.raises(ValueError, match="K values"):
        D.ssim_dp(a, a, K=(0.0, 0.03))
