"""The fused loss kernels inside a captured CUDA graph.

The kernels are launched with programmatic-dependent-launch attributes, TMA tensor maps in
their parameters and a per-stream reduction workspace; a graph captured from the forward
and backward calls must replay them with the results of eager execution, bit for bit,
and keep the workspace self-cleaning across replays.
"""

import pytest
import torch

from fussim_b200 import synthetic
from fussim_b200.functional import _ensure_cuda_extension

pytestmark = pytest.mark.gpu


def test_graph_replay_matches_eager():
    ext = _ensure_cuda_extension()
    a, b = synthetic.pair_noise((2, 3, 96, 200), 0.1, seed=5)
    a, b = a.cuda(), b.cuda()
    scale = 1.0 / a.numel()
    go = torch.ones((), device="cuda")

    def step():
        out, parts, _ = ext.loss_forward(a, b, 11, 1e-4, 9e-4, False, False, True, 1, False,
                                         scale)
        grad = ext.loss_backward(go, a, b, parts, 11, False, scale, 0)
        return out, grad

    eager = step()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # warm-up on the capture stream (its workspace is created here)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        captured = step()
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(captured[0], eager[0])
        assert torch.equal(captured[1], eager[1])
