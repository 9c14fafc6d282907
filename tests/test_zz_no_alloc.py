"""fssim_forward_noalloc, called through the C ABI, against fssim_forward.

fssim_forward_noalloc exists for callers that cannot allocate GPU memory — plugins whose
host application owns all device memory, real-time loops with a fixed memory budget,
bindings with no device allocator — so it keeps its reduction scratch in a fixed array
inside the library. This test calls it twice in a row (the array keeps the first call's
contents, which the entry point must clear) and compares every output with the regular
entry point run on a caller-provided workspace, within the parity tolerance used by the
other tests (1e-5). It also checks the batch limit is rejected with a clear error.

This file is named to be collected last, so a run that stops at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""

import ctypes
import os

import pytest
import torch

from fussim_b200 import synthetic

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "fussim_b200", "libfussim_b200.so")
MAX_IMAGES = 4096  # FSSIM_NOALLOC_MAX_IMAGES in include/fussim_b200.h


class ForwardArgs(ctypes.Structure):
    """Mirror of fssim_forward_args (include/fussim_b200.h)."""

    _fields_ = [
        ("dtype", ctypes.c_int32), ("partial_dtype", ctypes.c_int32),
        ("B", ctypes.c_int64), ("C", ctypes.c_int64), ("H", ctypes.c_int64),
        ("W", ctypes.c_int64),
        ("window_size", ctypes.c_int32), ("valid", ctypes.c_int32), ("clamp", ctypes.c_int32),
        ("train", ctypes.c_int32), ("reduce", ctypes.c_int32),
        ("C1", ctypes.c_float), ("C2", ctypes.c_float), ("out_scale", ctypes.c_float),
        ("img1", ctypes.c_void_p), ("img2", ctypes.c_void_p), ("ssim_map", ctypes.c_void_p),
        ("partials", ctypes.c_void_p), ("out", ctypes.c_void_p), ("image_sums", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("l1_weight", ctypes.c_float), ("out_offset", ctypes.c_float),
    ]


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    torch.cuda.init()
    lib = ctypes.CDLL(LIB)
    for name in ("fssim_forward", "fssim_forward_noalloc"):
        f = getattr(lib, name)
        f.argtypes = [ctypes.POINTER(ForwardArgs), ctypes.c_void_p]
        f.restype = ctypes.c_int
    lib.fssim_forward_workspace_bytes.argtypes = [ctypes.c_int64]
    lib.fssim_forward_workspace_bytes.restype = ctypes.c_size_t
    lib.fssim_last_error.restype = ctypes.c_char_p
    return lib


def _run(lib, fn_name, a, b, reduce, valid, workspace=None):
    B, C, H, W = a.shape
    dev = a.device
    partials = torch.empty((3, B, C, H, W), device=dev, dtype=torch.float32)
    out = torch.empty(1 if reduce == 1 else B, device=dev, dtype=torch.float32)
    sums = torch.empty(B, device=dev, dtype=torch.float64)
    h = 5 if valid else 0
    count = C * max(H - 2 * h, 0) * max(W - 2 * h, 0) * (B if reduce == 1 else 1)
    args = ForwardArgs(
        dtype=0, partial_dtype=0, B=B, C=C, H=H, W=W, window_size=11, valid=int(valid), clamp=0,
        train=1, reduce=reduce, C1=0.01**2, C2=0.03**2, out_scale=1.0 / count,
        img1=a.data_ptr(), img2=b.data_ptr(), ssim_map=None, partials=partials.data_ptr(),
        out=out.data_ptr(), image_sums=sums.data_ptr(),
        workspace=None if workspace is None else workspace.data_ptr(),
        workspace_bytes=0 if workspace is None else workspace.numel() * 8)
    st = getattr(lib, fn_name)(ctypes.byref(args), torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.fssim_last_error().decode()
    torch.cuda.synchronize()
    return out, sums, partials


@pytest.mark.parametrize("reduce,valid", [(1, False), (2, True)])
def test_noalloc_matches_forward_twice(lib, reduce, valid):
    a, b = synthetic.pair_noise((3, 2, 70, 133), 0.1, seed=41)
    a, b = a.cuda(), b.cuda()
    ws_bytes = lib.fssim_forward_workspace_bytes(3)
    workspace = torch.zeros((ws_bytes + 7) // 8, device="cuda", dtype=torch.int64)
    ref = _run(lib, "fssim_forward", a, b, reduce, valid, workspace)
    for _ in range(2):  # the second call starts from the first call's leftovers
        got = _run(lib, "fssim_forward_noalloc", a, b, reduce, valid)
        for g, r in zip(got, ref):
            assert (g.double() - r.double()).abs().max().item() <= 1e-5 * max(
                1.0, r.double().abs().max().item())
    # a different batch size right after: accumulators of the old batch must not leak in
    a2, b2 = a[:2].contiguous(), b[:2].contiguous()
    ref2 = _run(lib, "fssim_forward", a2, b2, reduce, valid, workspace)
    got2 = _run(lib, "fssim_forward_noalloc", a2, b2, reduce, valid)
    assert (got2[0].double() - ref2[0].double()).abs().max().item() <= 1e-5


def test_noalloc_rejects_oversized_batch(lib):
    args = ForwardArgs(dtype=0, partial_dtype=0, B=MAX_IMAGES + 1, C=1, H=8, W=8, window_size=11,
                       reduce=1, C1=1e-4, C2=9e-4, out_scale=1.0)
    st = lib.fssim_forward_noalloc(ctypes.byref(args), None)
    assert st == 5  # FSSIM_ERR_WORKSPACE
    assert b"at most 4096 images" in lib.fssim_last_error()


def test_no_device_side_failures_recorded(lib):
    """After every GPU test of the session, no kernel has reported a staging timeout."""
    lib.fssim_poll_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.c_int]
    lib.fssim_poll_device_error.restype = ctypes.c_int
    code = ctypes.c_uint(123)
    assert lib.fssim_poll_device_error(ctypes.byref(code), 0) == 0, lib.fssim_last_error().decode()
    assert code.value == 0
