"""The batch-sharded API on a one-rank NCCL group (one GPU).

A child process forms a world of one rank over NCCL on cuda:0 and runs the sharded entry
points next to their single-GPU counterparts on the same inputs:

* ``fused_ssim_dp`` goes through the peer mailboxes (the Python set-up of
  ``fussim_b200.distributed``: the same-host check, the IPC handle exchange, the published
  sum and the gather kernel, launched by the forward or, with ``async_op``, by ``wait()``
  after the backward or by the next step's call);
  its value must equal ``fused_ssim`` to FP32 rounding of the final scale and its gradient
  bitwise;
* ``ssim_dp`` goes through NCCL collectives (an all-reduce of the shard sum, or an
  all-gather of the per-image vector); value and gradient must equal ``ssim`` bitwise,
  with the clamp of ``nonnegative_ssim`` and per-image weights in the loss.

The multi-rank arithmetic of the same host code is covered on 2 gloo ranks by
test_distributed_cpu.py and on 2 GPUs by test_dp_gpu.py.
"""

import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPE = (3, 3, 96, 200)
WEIGHTS = (1.0, -2.0, 0.5)
MSSSIM_CASES = [(True, False), (False, False), (True, True), (False, True)]


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, queue):
    import torch.distributed as dist

    import fussim_b200 as fb
    from fussim_b200 import distributed as D
    from fussim_b200 import synthetic

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    res = {}
    try:
        _run(res, dev, fb, D, synthetic)
    except Exception:  # reported to the parent, which fails the tests with it
        res["error"] = traceback.format_exc()
    finally:
        dist.destroy_process_group()
    queue.put(res)


def _run(res, dev, fb, D, synthetic):
    a, b = synthetic.pair_noise(SHAPE, 0.1, seed=41)
    a, b = a.to(dev), b.to(dev)
    for padding in ("same", "valid"):
        for async_op in (False, True):
            # three steps in a row: with async_op the gather is launched by wait() (last
            # step) or by the next step's call (earlier steps)
            for it in range(3):
                x = a.clone().requires_grad_(True)
                if async_op:
                    v, work = D.fused_ssim_dp(x, b, padding=padding, async_op=True)
                    v.backward()
                    if it == 2:
                        work.wait()
                else:
                    v = D.fused_ssim_dp(x, b, padding=padding)
                    v.backward()
            y = a.clone().requires_grad_(True)
            r = fb.fused_ssim(y, b, padding=padding)
            r.backward()
            torch.cuda.synchronize()
            res[("fused", padding, async_op)] = (v.item(), r.item(),
                                                 bool(torch.equal(x.grad, y.grad)))
    b2 = (1.0 - b) * 0.5 + 0.5 * a    # partly anti-correlated: the clamp is exercised
    w = torch.tensor(WEIGHTS, device=dev)
    for size_average, nonneg in MSSSIM_CASES:
        out = []
        for fn in (D.ssim_dp, fb.ssim):
            x = a.clone().requires_grad_(True)
            v = fn(x, b2, data_range=1.0, size_average=size_average,
                   nonnegative_ssim=nonneg)
            (v if size_average else (v * w).sum()).backward()
            with torch.no_grad():
                v_ng = fn(x, b2, data_range=1.0, size_average=size_average,
                          nonnegative_ssim=nonneg)
            out.append((v.detach().cpu().numpy().copy(), v_ng.cpu().numpy().copy(),
                        x.grad.cpu().numpy().copy()))
        res[("msssim", size_average, nonneg)] = out
    res["errors"] = fb.poll_device_error(clear=True)
    D.release_mailboxes()
    torch.cuda.synchronize()


@pytest.fixture(scope="module")
def one_rank():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = mp.start_processes(_worker, args=(_free_port(), queue), nprocs=1, join=False,
                               start_method="spawn")
    res = queue.get(timeout=300)
    while not procs.join(timeout=120):
        pass
    assert "error" not in res, res["error"]
    return res


@pytest.mark.parametrize("padding", ["same", "valid"])
@pytest.mark.parametrize("async_op", [False, True])
def test_fused_ssim_dp_one_rank_matches_fused_ssim(one_rank, padding, async_op):
    v, r, grads_equal = one_rank[("fused", padding, async_op)]
    assert abs(v - r) <= 1e-7
    assert grads_equal


@pytest.mark.parametrize("size_average,nonneg", MSSSIM_CASES)
def test_ssim_dp_one_rank_matches_ssim(one_rank, size_average, nonneg):
    (v, v_ng, g), (r, r_ng, h) = one_rank[("msssim", size_average, nonneg)]
    assert v.shape == r.shape == (() if size_average else (SHAPE[0],))
    assert np.array_equal(v, r) and np.array_equal(v_ng, r_ng)
    assert np.array_equal(g, h)


def test_one_rank_run_left_no_device_error(one_rank):
    assert one_rank["errors"] == 0
