"""Batch-sharded SSIM over several GPUs (one process per GPU, torch.distributed).

Images are independent, so each rank computes the SSIM sum of its own shard of the batch
with the fused forward kernel; the only exchange is that scalar. The backward needs no
exchange: d(mean)/d(map) = 1/N_global is known from the shard shapes, so each rank's
gradient is local.

On one node with NCCL (GPUs), the scalar does not go through a collective call: the
forward kernel's last CTA stores the rank's sum into every rank's mailbox over NVLink
(CUDA IPC mappings set up once per group), and a one-warp gather kernel sums the world
values in rank order. A step then costs two kernel launches on the host, where an
all-reduce call costs about 35 us of host time, more than the kernels of a 1080p step
leave. Elsewhere (gloo, or more than 8 ranks) the sum is all-reduced with torch.distributed.

Failure behaviour: the gather waits at most 10 s (``set_gather_timeout``) for the other
ranks' sums; on time-out that step's value is NaN and a device
flag is set, which ``fussim_b200.check_device_errors()`` turns into a RuntimeError. A rank
expected to fall further behind (checkpointing, evaluation) should meet the others at a
host-side barrier first. On the ``dist.all_reduce`` path, the process group's own timeout
applies.

The reference has no distributed path; this is the engine's data-parallel form of
``fused_ssim`` (fussim/__init__.py:451-580): the value equals ``fused_ssim`` of the
concatenated global batch.
"""

from __future__ import annotations

import socket

import torch
import torch.distributed as dist

from . import functional as F

_count_cache: dict = {}
_mailboxes: dict = {}


def set_gather_timeout(seconds: float) -> None:
    """How long the peer exchange waits for the other ranks' sums before it gives up
    (default 10 s; ``seconds <= 0`` restores it). Process-wide; applies to later steps."""
    us = int(seconds * 1e6) if seconds > 0 else 0
    F._ensure_cuda_extension().set_gather_timeout_us(us)


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


class _Mailboxes:
    """This rank's mailbox and the peers' mailboxes mapped into this process (CUDA IPC)."""

    def __init__(self, group, device):
        ext = F._ensure_cuda_extension()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        with torch.cuda.device(device):
            self.local = ext.dp_mailbox_alloc(self.world)
            handle = ext.ipc_get_handle(self.local)
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=group)
            self.ptrs = [self.local if r == self.rank else ext.ipc_open_handle(h)
                         for r, h in enumerate(handles)]
        self.seq = 0
        # the deferred gather of an asynchronous step (a _LazyGather), launched by its wait()
        # or before this rank's next sharded forward: a rank publishes step k+1 only after
        # its own gather of step k, which keeps every peer within the two slot sets
        self.pending = None
        dist.barrier(group=group)  # every rank has mapped every mailbox before step 1

    def release(self):
        ext = F._ensure_cuda_extension()
        if self.pending is not None:
            self.pending.wait()
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                ext.ipc_close_handle(p)
        ext.dp_mailbox_free(self.local)
        self.ptrs = []


def _host_identity() -> str:
    """This machine as seen by the other ranks: host name plus the kernel's boot id, so
    containers that share a host name on different machines are told apart."""
    try:
        with open("/proc/sys/kernel/random/boot_id") as f:
            boot = f.read().strip()
    except OSError:
        boot = ""
    return f"{socket.gethostname()}/{boot}"


def _one_host(group) -> bool:
    """True when every rank of the group runs on this machine (CUDA IPC needs that)."""
    ids = [None] * dist.get_world_size(group)
    dist.all_gather_object(ids, _host_identity(), group=group)
    return len(set(ids)) == 1


def _mailboxes_for(group, device):
    """The group's mailboxes (created on first use), or None where the peer path is not
    available: a backend other than NCCL, more than 8 ranks, or ranks on several machines
    (decided once per group, collectively, on its first sharded step)."""
    if dist.get_backend(group) != "nccl" or dist.get_world_size(group) > 8:
        return None
    key = (id(group), device.index)
    if key not in _mailboxes:
        _mailboxes[key] = _Mailboxes(group, device) if _one_host(group) else None
    return _mailboxes[key]


def release_mailboxes():
    """Unmap and free every group's mailboxes. Every rank of each group that ran a sharded
    step must call it, after its last sharded step and before destroy_process_group (the
    barrier on that group keeps a rank from freeing its mailbox while a peer may still write
    into it)."""
    for mb in list(_mailboxes.values()):
        if mb is None:
            continue
        dist.barrier(group=mb.group)
        mb.release()
    _mailboxes.clear()


class _Done:
    """Handle of an exchange already ordered on the current stream."""

    def wait(self):
        return True

    def is_completed(self):
        return True


class _LazyGather:
    """Handle of a peer exchange whose gather kernel is not launched yet.

    ``wait()`` launches it on the current stream, after whatever the caller queued since the
    forward (typically the backward, which then does not wait for the other ranks'
    forwards); the next sharded forward of the same group launches it first if ``wait()``
    was not called. No host synchronisation either way."""

    def __init__(self, mb, out, scale, seq):
        self._mb = mb
        self._args = (out, scale, seq)
        mb.pending = self

    def wait(self):
        if self._args is not None:
            out, scale, seq = self._args
            self._args = None
            mb = self._mb
            if mb.pending is self:
                mb.pending = None
            F._ensure_cuda_extension().dp_gather(out, scale, mb.world, mb.rank, seq, mb.ptrs)
        return True

    def is_completed(self):
        return self._args is None


def _local_forward(a, b, window_size, C1, C2, valid, train, scale, clamp=False,
                   per_image=False):
    """Local shard: (out, partials). out = local_sum * scale (one value), or with
    ``per_image`` the (B_r,) vector of per-image sums * scale. Runs the fused CUDA kernel;
    ``clamp`` clamps the map at 0 before reducing (nonnegative_ssim)."""
    ext = F._ensure_cuda_extension()
    reduce = F._REDUCE_PER_IMAGE if per_image else F._REDUCE_SCALAR
    out, partials, _ = ext.loss_forward(a, b, window_size, C1, C2, valid, clamp, train, reduce,
                                        False, scale)
    return out, partials


def _local_backward(grad_out, a, b, partials, window_size, scale, grad_dtype, per_image=False):
    ext = F._ensure_cuda_extension()
    return ext.loss_backward(grad_out, a, b, partials, window_size, per_image, scale,
                             grad_dtype)


def _peer_forward(a, b, window_size, valid, train, scale, mb):
    """Local shard forward that publishes its sum, then the gather: out = global mean."""
    ext = F._ensure_cuda_extension()
    if mb.pending is not None:
        mb.pending.wait()
    mb.seq += 1
    out, partials = ext.loss_forward_dp(a, b, window_size, 0.01**2, 0.03**2, valid, train,
                                        scale, mb.world, mb.rank, mb.seq, mb.ptrs)
    ext.dp_gather(out, scale, mb.world, mb.rank, mb.seq, mb.ptrs)
    return out, partials


def _sharded_forward(a, b, window_size, valid, train, scale, group, works):
    mb = _mailboxes_for(group, a.device) if a.is_cuda else None
    if mb is not None:
        out, partials = _peer_forward(a, b, window_size, valid, train, scale, mb)
        works.append(_Done())
        return out, partials
    out, partials = _local_forward(a, b, window_size, 0.01**2, 0.03**2, valid, train, scale)
    works.append(dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group, async_op=True))
    return out, partials


class _ShardedSSIM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, img1, img2, window_size, valid, half, scale, group, works):
        a, b = F._kernel_inputs(img1, img2, half)
        out, partials = _sharded_forward(a, b, window_size, valid, True, scale, group, works)
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
    returns ``(value, work)`` without waiting for the exchange: the local backward can run
    meanwhile, and ``work.wait()`` must be called before the value is read. (On the peer
    path ``wait`` launches the gather of the shard sums on the current stream, after the
    backward, so the backward does not wait for the other ranks; there is no host
    synchronisation.) Every rank must make the same sequence of calls.
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
    mb = _mailboxes_for(group, img1.device) if (train and img1.is_cuda) else None
    if mb is not None:
        # peer path: the C++ autograd function of the extension (forward publishes the shard
        # sum, backward is local); the gather of the shard sums follows on this stream, or,
        # with async_op, on the mailboxes' stream so that the backward need not wait for the
        # other ranks' forwards
        ext = F._ensure_cuda_extension()
        if mb.pending is not None:
            mb.pending.wait()
        mb.seq += 1
        chain = scale if scale != float("inf") else 0.0
        out = ext.fused_loss_dp(img1, img2, window_size, valid, half, scale, chain, mb.world,
                                mb.rank, mb.seq, mb.ptrs, gather=not async_op)
        works.append(_LazyGather(mb, out, scale, mb.seq) if async_op else _Done())
    elif train:
        out = _ShardedSSIM.apply(img1, img2, window_size, valid, half, scale, group, works)
    else:
        a, b = F._kernel_inputs(img1, img2, half)
        out, _ = _sharded_forward(a, b, window_size, valid, False, scale, group, works)
    if async_op:
        return out, works[0]
    works[0].wait()
    return out


# ------------------------------------------------------------------------------------
# pytorch-msssim form over a sharded batch
# ------------------------------------------------------------------------------------

def shard_sizes(local_batch: int, group=None) -> list:
    """Every rank's batch size, in rank order (one all-gather per distinct local size,
    cached)."""
    key = ("B", local_batch, id(group))
    if key not in _count_cache:
        dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
            else torch.device("cpu")
        t = torch.tensor([local_batch], dtype=torch.int64, device=dev)
        parts = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
        dist.all_gather(parts, t, group=group)
        _count_cache[key] = [int(x.item()) for x in parts]
    return _count_cache[key]


def _gather_per_image(local, sizes, group):
    """Concatenation in rank order of every rank's (B_r,) vector (padded to the largest
    shard for the all-gather, then trimmed)."""
    width = max(sizes)
    buf = local.new_zeros(width)
    buf[:local.numel()] = local
    parts = [torch.empty_like(buf) for _ in sizes]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([p[:n] for p, n in zip(parts, sizes)])


class _ShardedMsssim(torch.autograd.Function):
    """Forward: the local fused kernel (clamp and per-image reduction in the kernel), then
    the exchange (a sum for the global mean, an all-gather of the per-image vectors).
    Backward: local; with per-image values the rank's slice of the upstream gradient."""

    @staticmethod
    def forward(ctx, img1, img2, C1, C2, window_size, clamp, per_image, half, scale, group):
        a, b = F._kernel_inputs(img1, img2, half)
        out, partials = _local_forward(a, b, window_size, C1, C2, True, True, scale, clamp,
                                       per_image)
        if per_image:
            sizes = shard_sizes(a.shape[0], group)
            rank = dist.get_rank(group)
            ctx.lo, ctx.n = sum(sizes[:rank]), sizes[rank]
            out = _gather_per_image(out, sizes, group)
        else:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
        ctx.save_for_backward(a, b, partials)
        ctx.window_size = window_size
        ctx.per_image = per_image
        ctx.scale = scale if scale != float("inf") else 0.0
        ctx.grad_dtype = F._DTYPE_CODE.get(img1.dtype, 0)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        a, b, partials = ctx.saved_tensors
        if ctx.per_image:
            grad_out = grad_out[ctx.lo:ctx.lo + ctx.n]
        grad = _local_backward(grad_out, a, b, partials, ctx.window_size, ctx.scale,
                               ctx.grad_dtype, ctx.per_image)
        return (grad,) + (None,) * 9


def ssim_dp(X, Y, data_range=255, size_average=True, win_size=11, win_sigma=1.5, win=None,
            K=(0.01, 0.03), nonnegative_ssim=False, group=None):
    """``fussim_b200.ssim`` (pytorch-msssim form, 'valid' padding) of the batch formed by
    every rank's (X, Y) shard.

    With ``size_average=True`` every rank gets the global mean over all shards' pixels (one
    all-reduce of the shard sums); with ``size_average=False`` every rank gets the (B,)
    vector of per-image values of the whole batch in rank order (one all-gather of the
    per-image vectors), and the gradient reaching this rank's X is that of its own images'
    entries. The argument checks and their messages are the reference's ``ssim``
    (fussim/__init__.py:636-658). Every rank must make the same sequence of calls.
    """
    C1, C2 = F._msssim_constants(data_range, win_size, win_sigma, win, K)
    half = torch.is_autocast_enabled()
    if not half:
        X, Y = F._float_path_inputs(X, Y)
    per_image = not size_average
    if per_image:
        scale = F._inv(F._count(tuple(X.shape), win_size, True, True))
    else:
        scale = F._inv(global_count(F._count(tuple(X.shape), win_size, True, False), group))
    if torch.is_grad_enabled() and X.requires_grad:
        return _ShardedMsssim.apply(X, Y, C1, C2, win_size, bool(nonnegative_ssim), per_image,
                                    half, scale, group)
    a, b = F._kernel_inputs(X, Y, half)
    out, _ = _local_forward(a, b, win_size, C1, C2, True, False, scale, bool(nonnegative_ssim),
                            per_image)
    if per_image:
        return _gather_per_image(out, shard_sizes(a.shape[0], group), group)
    dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
    return out
