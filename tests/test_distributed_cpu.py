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


def _oracle_local_forward(a, b, window_size, C1, C2, valid, train, scale):
    """Stand-in for the fused forward kernel: (local sum * scale, masked partials)."""
    m, p0, p1, p2 = O.ssim_map_and_partials(a, b, window_size, C1, C2)
    mask = _crop_mask(a.shape, window_size, valid)
    out = torch.tensor([float((m * mask).sum()) * scale], dtype=torch.float32)
    partials = torch.stack([p0 * mask, p1 * mask, p2 * mask]).to(torch.float32)
    return out, partials


def _oracle_local_backward(grad_out, a, b, partials, window_size, scale, grad_dtype):
    """Stand-in for the fused backward kernel: dL/dimg1 with dL/dmap = grad_out * scale."""
    dl = torch.full(a.shape, float(grad_out) * scale, dtype=torch.float64)
    g = O.backward_closed_form(a, b, dl, tuple(partials.to(torch.float64)), window_size)
    return g.to(torch.float32)


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


def test_sharded_argument_errors():
    from fussim_b200 import distributed as D

    a = torch.rand(1, 3, 16, 16)
    with pytest.raises(ValueError, match="padding"):
        D.fused_ssim_dp(a, a, padding="reflect")
    with pytest.raises(ValueError, match="window_size"):
        D.fused_ssim_dp(a, a, window_size=5)
