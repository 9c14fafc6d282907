"""The batch-sharded path on 2 GPUs (NCCL), against the single-GPU fused loss.

Runs only where two GPUs are visible. Two child processes (one per GPU) each hold one shard
of a seeded global batch; the value of fused_ssim_dp must equal fused_ssim of the whole
batch on one GPU, and each rank's gradient the matching slice of its gradient. NVLink
SHARP reductions are switched off (NCCL_NVLS_ENABLE=0). The shard sums travel through the
peer mailboxes (CUDA IPC over NVLink); NCCL carries only the one-time set-up (the pixel
count and the exchange of the IPC handles). ``ssim_dp(size_average=False)`` must give every
rank the whole batch's per-image vector of ``ssim`` and each rank the slice of the gradient
of a per-image weighted loss.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHARDS = (1, 2)
SHAPE = (3, 96, 200)
WEIGHTS = (1.0, -2.0, 0.5)   # per-image weights of the ssim_dp loss


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _global_pair():
    from fussim_b200 import synthetic

    return synthetic.pair_noise((sum(SHARDS),) + SHAPE, 0.1, seed=31)


def _worker(rank, port, queue):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from fussim_b200 import distributed as D

        a_all, b_all = _global_pair()
        lo = sum(SHARDS[:rank])
        out = {}
        for padding in ("same", "valid"):
            # several steps, asynchronous (gather on a side stream) and synchronous mixed:
            # every one must give the same value and gradient
            vals, grads = [], []
            for it in range(5):
                a = a_all[lo:lo + SHARDS[rank]].to(dev).requires_grad_(True)
                b = b_all[lo:lo + SHARDS[rank]].to(dev)
                if it % 2 == 0:
                    v, work = D.fused_ssim_dp(a, b, padding=padding, async_op=True)
                    v.backward()
                    work.wait()
                else:
                    v = D.fused_ssim_dp(a, b, padding=padding)
                    v.backward()
                vals.append(v.detach().clone())
                grads.append(a.grad)
            torch.cuda.synchronize()
            assert all(torch.equal(g, grads[0]) for g in grads)
            out[padding] = ([float(x) for x in vals], a.grad.cpu().numpy().copy())
        # the peer path (mailboxes over CUDA IPC) must have been used, not a collective
        out["peer"] = len(D._mailboxes) == 1
        # pytorch-msssim form over NCCL: per-image vector of the whole batch on every rank
        a = a_all[lo:lo + SHARDS[rank]].to(dev).requires_grad_(True)
        b = b_all[lo:lo + SHARDS[rank]].to(dev)
        v = D.ssim_dp(a, b, data_range=1.0, size_average=False)
        (v * torch.tensor(WEIGHTS, device=dev)).sum().backward()
        out["per_image"] = (v.detach().cpu().numpy().copy(), a.grad.cpu().numpy().copy())
        D.release_mailboxes()
        queue.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_dp_two_gpus_matches_single_gpu():
    import fussim_b200 as fb

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = mp.start_processes(_worker, args=(_free_port(), queue), nprocs=2, join=False,
                               start_method="spawn")
    res = {}
    for _ in range(2):
        rank, r = queue.get(timeout=180)
        res[rank] = r
    while not procs.join(timeout=120):
        pass
    a_all, b_all = _global_pair()
    assert res[0]["peer"] and res[1]["peer"]
    for padding in ("same", "valid"):
        x = a_all.cuda().requires_grad_(True)
        v = fb.fused_ssim(x, b_all.cuda(), padding=padding)
        v.backward()
        g = x.grad.cpu()
        for rank in range(2):
            vals, grad = res[rank][padding]
            assert all(abs(val - v.item()) <= 1e-6 for val in vals)
            lo = sum(SHARDS[:rank])
            ref = g[lo:lo + SHARDS[rank]]
            assert (torch.from_numpy(grad) - ref).abs().max().item() <= 1e-5 * ref.abs().max().item()
    x = a_all.cuda().requires_grad_(True)
    v = fb.ssim(x, b_all.cuda(), data_range=1.0, size_average=False)
    (v * torch.tensor(WEIGHTS, device=v.device)).sum().backward()
    g = x.grad.cpu()
    for rank in range(2):
        vals, grad = res[rank]["per_image"]
        assert (torch.from_numpy(vals) - v.detach().cpu()).abs().max().item() <= 1e-6
        lo = sum(SHARDS[:rank])
        ref = g[lo:lo + SHARDS[rank]]
        assert (torch.from_numpy(grad) - ref).abs().max().item() <= 1e-5 * ref.abs().max().item()
