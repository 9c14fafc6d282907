"""Host-side behaviour of the drop-in API and the C ABI (runs without a GPU).

The reference raises before touching the GPU for bad parameters (fussim/__init__.py:503-547,
636-658, 739-752); these checks run here on CPU tensors. The C-ABI library must load and
export every function declared in include/fussim_b200.h; only argument-validation paths
that return before any CUDA call are exercised here.
"""

import ctypes
import os
import re

import pytest
import torch

import fussim_b200 as fb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fussim_b200.h")
LIB = os.path.join(ROOT, "fussim_b200", "libfussim_b200.so")


def test_public_names():
    assert fb.SUPPORTED_WINDOW_SIZES == (7, 9, 11)
    for name in ("fused_ssim", "ssim", "SSIM", "FusedSSIMMap", "FusedSSIMMapFP16",
                 "__version__", "get_build_info", "check_compatibility",
                 "SUPPORTED_WINDOW_SIZES"):
        assert name in fb.__all__ and hasattr(fb, name)
    info = fb.get_build_info()
    assert info["arch"] == "sm_100a" and info["is_prebuilt"] is False
    ok, issues = fb.check_compatibility(warn=False)
    assert isinstance(ok, bool) and isinstance(issues, list)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-CUDA error path")
def test_fused_ssim_requires_cuda():
    a = torch.rand(1, 3, 16, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        fb.fused_ssim(a, a)


@pytest.mark.parametrize("kwargs,match", [
    (dict(win_size=5), "win_size"),
    (dict(win_sigma=1.0), "win_sigma"),
    (dict(win=torch.ones(1, 1, 11, 11)), "win"),
    (dict(K=(0.01,)), "K"),
    (dict(K=(0, 0.03)), "K"),
    (dict(K=(0.01, 1.5)), "K"),
])
def test_ssim_parameter_validation(kwargs, match):
    a = torch.rand(1, 3, 16, 16)
    with pytest.raises(ValueError, match=match):
        fb.ssim(a, a, **kwargs)


@pytest.mark.parametrize("kwargs,match", [
    (dict(win_size=5), "win_size"),
    (dict(win_sigma=2.0), "win_sigma"),
    (dict(spatial_dims=3), "spatial_dims"),
    (dict(K=(0.5, 1.0)), "K"),
])
def test_module_parameter_validation(kwargs, match):
    with pytest.raises(ValueError, match=match):
        fb.SSIM(**kwargs)


def test_module_stores_parameters():
    m = fb.SSIM(data_range=1.0, size_average=False, win_size=7, channel=5, K=[0.02, 0.04],
                nonnegative_ssim=True)
    assert (m.data_range, m.size_average, m.win_size, m.K, m.nonnegative_ssim) == \
        (1.0, False, 7, (0.02, 0.04), True)


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(fssim_\w+)\s*\(", text, re.M)))


def test_cabi_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    names = _declared_functions()
    assert len(names) >= 11, names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/fussim_b200.h but not exported"


def test_cabi_host_only_paths():
    lib = ctypes.CDLL(LIB)
    lib.fssim_status_string.restype = ctypes.c_char_p
    lib.fssim_last_error.restype = ctypes.c_char_p
    lib.fssim_version.restype = ctypes.c_char_p
    lib.fssim_forward_workspace_bytes.restype = ctypes.c_size_t
    lib.fssim_forward_workspace_bytes.argtypes = [ctypes.c_int64]
    assert lib.fssim_status_string(0) == b"success"
    assert lib.fssim_version().decode() == fb.__version__
    assert lib.fssim_forward_workspace_bytes(4) >= 4 * 8
    # a bad window size is rejected before any CUDA call, with the reference's message
    f = lib.fssim_fusedssim
    f.argtypes = [ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_void_p]
    st = f(5, 1e-4, 9e-4, None, None, 1, 1, 8, 8, 0, None, None, None, None, None)
    assert st == 1
    assert lib.fssim_last_error() == b"window_size must be 7, 9, or 11, got 5"
    # an empty batch is a no-op that succeeds without touching the GPU
    assert f(11, 1e-4, 9e-4, None, None, 0, 3, 8, 8, 1, None, None, None, None, None) == 0
    # negative sizes are a shape error
    assert f(11, 1e-4, 9e-4, None, None, -1, 3, 8, 8, 1, None, None, None, None, None) == 2
    # the reserved-SM count is host state: negative counts are an argument error
    lib.fssim_set_reserved_sms.argtypes = [ctypes.c_int]
    assert lib.fssim_set_reserved_sms(-1) == 7  # FSSIM_ERR_ARGUMENT
    assert lib.fssim_last_error() == b"reserved SM count must be >= 0"
    assert lib.fssim_set_reserved_sms(0) == 0
