"""Failure detection of the batch-sharded path, on gloo ranks on the CPU.

No GPU is involved: the failures are made on the host (a rank that raises, a rank that
exits between steps, a rank that never joins), and each rank's local forward and backward
are replaced by the float64 oracle as in test_distributed_cpu.py. What is checked is that
the surviving rank's next sharded step (or its process-group set-up) ends with an error
within the process group's short timeout instead of waiting for good, and that
``release_mailboxes`` synchronises only the ranks of the group that owns the mailboxes.
"""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

TIMEOUT_S = 4          # process-group timeout of the ranks
DEADLINE_S = 60        # a surviving rank must have seen its error well before this


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=TIMEOUT_S))


def _sharded_step(seed):
    from fussim_b200 import distributed as D
    from fussim_b200 import synthetic
    from tests import test_distributed_cpu as T

    D._local_forward = T._oracle_local_forward
    D._local_backward = T._oracle_local_backward
    a, b = synthetic.pair_noise((1, 3, 20, 24), 0.1, seed=seed)
    a.requires_grad_(True)
    v = D.fused_ssim_dp(a, b)
    v.backward()
    return float(v.detach())


def _put(queue, item):
    """Put and flush, so the item survives an os._exit right after."""
    queue.put(item)
    queue.close()
    queue.join_thread()


def _survivor_next_step(queue, rank):
    """Run step 2 on a rank whose peer has failed; report how it ended."""
    t0 = time.time()
    try:
        _sharded_step(2)
        _put(queue, (rank, "completed", time.time() - t0, ""))
    except Exception as e:  # noqa: BLE001 (any error type is the expected outcome)
        _put(queue, (rank, "error", time.time() - t0, f"{type(e).__name__}: {e}"[:200]))


def _worker_raises(rank, port, queue):
    _init(rank, 2, port)
    _sharded_step(1)
    if rank == 1:
        try:
            raise RuntimeError("rank 1 failed in its own code before step 2")
        except RuntimeError as e:
            _put(queue, (rank, "raised", 0.0, str(e)))
        # the failed rank stays alive without entering step 2 until the survivor has
        # given up, so only the process group's timeout can end the survivor's wait
        time.sleep(TIMEOUT_S + 8)
        os._exit(0)
    _survivor_next_step(queue, rank)
    os._exit(0)


def _worker_exits(rank, port, queue):
    _init(rank, 2, port)
    _sharded_step(1)
    if rank == 1:
        _put(queue, (rank, "exited", 0.0, ""))
        os._exit(0)  # leaves between steps, with nothing in flight
    _survivor_next_step(queue, rank)
    os._exit(0)


def _worker_init_timeout(rank, port, queue):
    # world_size 2, but rank 1 is never started
    t0 = time.time()
    try:
        _init(rank, 2, port)
        _put(queue, (rank, "completed", time.time() - t0, ""))
    except Exception as e:  # noqa: BLE001
        _put(queue, (rank, "error", time.time() - t0, f"{type(e).__name__}: {e}"[:200]))
    os._exit(0)


def _run(fn, nprocs):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = mp.start_processes(fn, args=(_free_port(), queue), nprocs=nprocs, join=False,
                               start_method="spawn")
    out = []
    t0 = time.time()
    try:
        while len(out) < nprocs and time.time() - t0 < DEADLINE_S + 60:
            try:
                out.append(queue.get(timeout=5))
            except Exception:  # noqa: BLE001 (queue.Empty: keep polling until the deadline)
                pass
    finally:
        for p in procs.processes:
            p.join(timeout=TIMEOUT_S + 30)
            if p.is_alive():
                p.kill()
    return {r[0]: r[1:] for r in out}


def test_rank_that_raises_ends_the_survivors_step():
    res = _run(_worker_raises, 2)
    assert res[1][0] == "raised"
    status, took, msg = res[0]
    assert status == "error", f"survivor did not fail: {res[0]}"
    assert took < DEADLINE_S, f"survivor waited {took:.1f} s"


def test_rank_that_exits_ends_the_survivors_step():
    res = _run(_worker_exits, 2)
    assert res[1][0] == "exited"
    status, took, msg = res[0]
    assert status == "error", f"survivor did not fail: {res[0]}"
    assert took < DEADLINE_S, f"survivor waited {took:.1f} s"


def test_init_process_group_times_out_without_peer():
    res = _run(_worker_init_timeout, 1)
    status, took, msg = res[0]
    assert status == "error", f"init did not fail: {res[0]}"
    assert took < DEADLINE_S, f"init waited {took:.1f} s"


class _FakeMailboxes:
    """Stands in for a group's CUDA IPC mailboxes (which need GPUs) in release_mailboxes."""

    def __init__(self, group):
        self.group = group
        self.released = False

    def release(self):
        self.released = True


def _worker_subgroup_release(rank, port, queue):
    _init(rank, 3, port)
    from fussim_b200 import distributed as D

    sub = dist.new_group([0, 1])  # every rank takes part in creating the subgroup
    if rank in (0, 1):
        D._mailboxes[(id(sub), 0)] = _FakeMailboxes(sub)
    t0 = time.time()
    try:
        D.release_mailboxes()  # rank 2 owns none and must not be waited for
        _put(queue, (rank, "released", time.time() - t0, ""))
    except Exception as e:  # noqa: BLE001
        _put(queue, (rank, "error", time.time() - t0, f"{type(e).__name__}: {e}"[:200]))
    if rank == 2:
        # enters no collective for longer than the timeout: a barrier of ranks 0 and 1 on
        # the whole world (rather than on their group) would time out meanwhile
        time.sleep(TIMEOUT_S + 3)
    os._exit(0)


def test_release_mailboxes_barriers_on_the_owning_group():
    res = _run(_worker_subgroup_release, 3)
    for rank in range(3):
        status, took, msg = res[rank]
        assert status == "released", f"rank {rank}: {res[rank]}"
        assert took < TIMEOUT_S, f"rank {rank} waited {took:.1f} s"
