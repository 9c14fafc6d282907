"""Host logic of the deferred peer gather (fussim_b200.distributed), on the CPU.

With ``fused_ssim_dp(..., async_op=True)`` on the peer path the forward only publishes the
rank's sum; the gather kernel is launched later, by ``work.wait()`` or, if the caller did
not wait, by the next sharded forward of the same group before it publishes again (a rank
must gather step k before it publishes step k+1, which keeps every peer within the two slot
sets of the mailboxes). ``release_mailboxes`` launches a still-pending gather before it
frees anything. The extension is replaced by a recorder: no GPU is involved, the test
checks which launches the host issues and in which order.
"""

import pytest

from fussim_b200 import distributed as D
from fussim_b200 import functional as F


class _Recorder:
    def __init__(self):
        self.calls = []

    def dp_gather(self, out, scale, world, rank, seq, ptrs):
        self.calls.append(("gather", out, seq))

    def loss_forward_dp(self, a, b, ws, C1, C2, valid, train, scale, world, rank, seq, ptrs):
        self.calls.append(("forward", None, seq))
        return f"out{seq}", f"partials{seq}"

    def ipc_close_handle(self, p):
        self.calls.append(("close", p, None))

    def dp_mailbox_free(self, p):
        self.calls.append(("free", p, None))


class _FakeMailboxes(D._Mailboxes):
    def __init__(self):  # no process group, no CUDA: only the fields the host logic uses
        self.world, self.rank, self.seq = 2, 0, 0
        self.local = 100
        self.ptrs = [100, 200]
        self.pending = None


@pytest.fixture
def rec(monkeypatch):
    r = _Recorder()
    monkeypatch.setattr(F, "_ensure_cuda_extension", lambda: r)
    return r


def test_wait_launches_the_gather_once(rec):
    mb = _FakeMailboxes()
    work = D._LazyGather(mb, "out1", 0.5, 1)
    assert mb.pending is work and not work.is_completed()
    assert work.wait() is True
    assert rec.calls == [("gather", "out1", 1)]
    assert mb.pending is None and work.is_completed()
    work.wait()
    assert rec.calls == [("gather", "out1", 1)]


def test_next_forward_gathers_the_pending_step_before_publishing(rec):
    mb = _FakeMailboxes()
    mb.seq = 1
    work = D._LazyGather(mb, "out1", 0.5, 1)
    out, partials = D._peer_forward(None, None, 11, False, False, 0.5, mb)
    assert (out, partials) == ("out2", "partials2")
    assert rec.calls == [("gather", "out1", 1), ("forward", None, 2), ("gather", "out2", 2)]
    assert work.is_completed() and mb.pending is None
    work.wait()  # already launched by the forward: nothing more
    assert len(rec.calls) == 3


def test_a_later_handle_does_not_clear_a_newer_pending_one(rec):
    mb = _FakeMailboxes()
    first = D._LazyGather(mb, "out1", 0.5, 1)
    first.wait()
    second = D._LazyGather(mb, "out2", 0.5, 2)
    first.wait()
    assert mb.pending is second
    second.wait()
    assert mb.pending is None
    assert [c[2] for c in rec.calls] == [1, 2]


def test_release_launches_a_pending_gather_before_freeing(rec):
    mb = _FakeMailboxes()
    D._LazyGather(mb, "out1", 0.5, 1)
    mb.release()
    assert rec.calls == [("gather", "out1", 1), ("close", 200, None), ("free", 100, None)]
    assert mb.pending is None and mb.ptrs == []
