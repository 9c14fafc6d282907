"""Batch-sharded SSIM over several GPUs (one process per GPU, torch.distributed + NCCL).

Images are independent, so each rank computes the SSIM sum of its own shard of the batch
with the fused forward kernel; the only exchange is one all-reduce of that scalar over
NVLink/NVSwitch. The backward needs no collective: d(mean)/d(map) = 1/N_global is known
from the shard shapes, so each rank's gradient is local.

The reference has no distributed path; this is the engine's data-parallel form of
``fused_ssim`` (fussim/__init__.py:451-580): the value equals ``fused_ssim`` of the
concatenated global batch.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import functional as F

_count_cache: dict = {}


def global_count(local_count: int, group=None) -> int:
    """Sum of the per-rank pixel counts (one all-reduce per distinct local count, cached)."""
    key = (local_count, id(group))
    if key not in _count_cache:
        dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
            else torch.device("cpu")
        t = torch.tensor([local_count], dtype=torch.int64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
        _count_cache[key] = int(t.item())
    return _count_cache[key]


def _local_forward(a, b, window_size, C1, C2, valid, train, scale):
    """Local shard: (out = local_sum * scale, partials). Runs the fused CUDA kernel."""
    ext = F._ensure_cuda_extension()
    out, partials, _ = ext.loss_forward(a, b, window_size, C1, C2, valid, False, train,
                                        F._REDUCE_SCALAR, False, scale)
    return out, partials


def _local_backward(grad_out, a, b, partials, window_size, scale, grad_dtype):
    ext = F._ensure_cuda_extension()
    return ext.loss_backward(grad_out, a, b, partials, window_size, False, scale, grad_dtype)


class _ShardedSSIM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, img1, img2, window_size, valid, half, scale, group, works):
        a, b = F._kernel_inputs(img1, img2, half)
        out, partials = _local_forward(a, b, window_size, 0.01**2, 0.03**2, valid, True, scale)
        works.append(dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group, async_op=True))
        ctx.save_for_backward(a, b, partials)
        ctx.window_size = window_size
        ctx.scale = scale if scale != float("inf") else 0.0
        ctx.grad_dtype = F._DTYPE_CODE.get(img1.dtype, 0)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        a, b, partials = ctx.saved_tensors
        grad = _local_backward(grad_out, a, b, partials, ctx.window_size, ctx.scale,
                               ctx.grad_dtype)
        return grad, None, None, None, None, None, None, None


def fused_ssim_dp(img1, img2, padding="same", train=True, window_size=11, group=None,
                  async_op=False):
    """Mean SSIM over the batch formed by every rank's (img1, img2) shard.

    Each rank passes its own (B_r, C, H, W) shard; the result (on every rank) equals
    ``fused_ssim`` of the concatenation of all shards. With ``async_op=True`` the call
    returns ``(value, work)`` without waiting for the all-reduce: the local backward can
    run meanwhile, and ``work.wait()`` must be called before the value is read.
    """
    if padding not in F.ALLOWED_PADDING:
        raise ValueError(f"padding must be one of {F.ALLOWED_PADDING}, but got '{padding}'")
    if window_size not in F.SUPPORTED_WINDOW_SIZES:
        raise ValueError(
            f"window_size must be one of {F.SUPPORTED_WINDOW_SIZES}, got {window_size}")
    valid = padding == "valid"
    n = global_count(F._count(tuple(img1.shape), window_size, valid, False), group)
    scale = F._inv(n)
    half = torch.is_autocast_enabled()
    train = train and torch.is_grad_enabled() and img1.requires_grad
    works: list = []
    if train:
        out = _ShardedSSIM.apply(img1, img2, window_size, valid, half, scale, group, works)
    else:
        a, b = F._kernel_inputs(img1, img2, half)
        out, _ = _local_forward(a, b, window_size, 0.01**2, 0.03**2, valid, False, scale)
        works.append(dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group, async_op=True))
    if async_op:
        return out, works[0]
    works[0].wait()
    return out
