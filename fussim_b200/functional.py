"""Public SSIM API over the sm_100a kernels.

Behaviour mirrors OpsiClear/fussim ``fussim/__init__.py`` (validation order and messages,
autocast dispatch, gradient to img1 only, FP32 results). The computation differs: the
scalar and per-image reductions are fused into the forward kernel, the backward folds the
upstream gradient in as a per-image scalar, and the valid crop and the clamp of
``nonnegative_ssim`` happen inside the kernels, so a forward+backward is two kernel
launches.
"""

from __future__ import annotations

import importlib
import os
import warnings

import torch

__version__ = "0.1.0"

# Window sizes with kernel instantiations (reference: fussim/__init__.py:31-32).
SUPPORTED_WINDOW_SIZES = (7, 9, 11)
ALLOWED_PADDING = ("same", "valid")

_REDUCE_SCALAR = 1
_REDUCE_PER_IMAGE = 2
_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_cuda_extension = None


def _ensure_cuda_extension():
    """Load the in-tree torch extension (``_C.so`` over ``libfussim_b200.so``).

    Raises ImportError when it has not been built: there is no fallback path.
    """
    global _cuda_extension
    if _cuda_extension is not None:
        return _cuda_extension
    try:
        _cuda_extension = importlib.import_module(__package__ + "._C")
    except ImportError as e:
        raise ImportError(
            "fussim_b200 CUDA extension is not built. Build it in-tree with\n"
            "    python -m fussim_b200.build\n"
            f"Original error: {e}"
        ) from e
    return _cuda_extension


def get_build_info():
    """How this package was built (keys of the reference's get_build_info, plus ``arch``)."""
    here = os.path.dirname(os.path.abspath(__file__))
    return {
        "version": __version__,
        "base_version": __version__,
        "build_torch_version": None,
        "build_cuda_version": None,
        "runtime_torch_version": torch.__version__.split("+")[0],
        "runtime_cuda_version": torch.version.cuda if torch.cuda.is_available() else None,
        "is_prebuilt": False,
        "arch": "sm_100a",
        "extension_built": os.path.exists(os.path.join(here, "_C.so"))
        and os.path.exists(os.path.join(here, "libfussim_b200.so")),
    }


def check_compatibility(warn=True):
    """Return (is_compatible, issues). The kernels are built for sm_100a (B200) only."""
    issues = []
    if torch.cuda.is_available():
        for i in range(torch.cuda.device_count()):
            major, minor = torch.cuda.get_device_capability(i)
            if (major, minor) != (10, 0):
                issues.append(
                    f"GPU {i} has compute capability {major}.{minor}; "
                    "fussim_b200 kernels are built for sm_100a (B200) only."
                )
    if warn:
        for issue in issues:
            warnings.warn(issue, RuntimeWarning, stacklevel=2)
    return len(issues) == 0, issues


_DEVICE_ERROR_BITS = {
    1: "a kernel's input staging did not complete within its bounded wait (the reduced "
       "outputs of that call are NaN; its per-pixel outputs are incomplete)",
    2: "the sharded exchange gave up waiting for another rank (that step's value is NaN)",
}


def poll_device_error(clear: bool = True) -> int:
    """Failures the kernels recorded on the current CUDA device since the last clear, as a
    bit set (0 = none; the bits are those of ``check_device_errors``). Synchronises with the
    device, so call it between steps (e.g. when a loss comes back NaN), not inside one."""
    return int(_ensure_cuda_extension().poll_device_error(bool(clear)))


def check_device_errors(clear: bool = True) -> None:
    """Raise RuntimeError if a kernel recorded a failure on the current CUDA device.

    The kernels never trap: a staging copy that does not arrive within its bounded wait, or
    a sharded exchange whose peer does not answer in time, ends the affected work, writes
    NaN to the reduced result and records a bit in a device flag. This reads (and by default
    clears) that flag.
    """
    code = poll_device_error(clear)
    if code:
        msgs = [m for bit, m in _DEVICE_ERROR_BITS.items() if code & bit]
        raise RuntimeError(f"fussim_b200 device error 0x{code:x}: " + "; ".join(msgs))


def _get_halo(window_size: int) -> int:
    return (window_size - 1) // 2


def _count(shape, window_size: int, valid: bool, per_image: bool) -> int:
    b, c, h, w = shape
    if valid:
        k = 2 * _get_halo(window_size)
        h, w = max(h - k, 0), max(w - k, 0)
    n = c * h * w
    return n if per_image else b * n


def _inv(n: int) -> float:
    return 1.0 / n if n > 0 else float("inf")


# ------------------------------------------------------------------------------------
# Reference-compatible map-producing autograd Functions
# ------------------------------------------------------------------------------------
class FusedSSIMMap(torch.autograd.Function):
    """SSIM map of (img1, img2) with gradient to img1 (reference: fussim/__init__.py:351-395).

    ``apply(C1, C2, img1, img2, padding="same", train=True, window_size=11)`` returns the
    per-pixel map (cropped by (window_size-1)/2 on every side for ``padding="valid"``).
    """

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda", cast_inputs=torch.float32)
    def forward(ctx, C1, C2, img1, img2, padding="same", train=True, window_size=11):
        ext = _ensure_cuda_extension()
        ssim_map, p0, p1, p2 = ext.fusedssim(window_size, C1, C2, img1, img2, train)
        h = _get_halo(window_size)
        if padding == "valid":
            ssim_map = ssim_map[:, :, h:-h, h:-h]
        ctx.save_for_backward(img1.detach(), img2, p0, p1, p2)
        ctx.C1, ctx.C2, ctx.padding, ctx.window_size = C1, C2, padding, window_size
        return ssim_map

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, opt_grad):
        ext = _ensure_cuda_extension()
        img1, img2, p0, p1, p2 = ctx.saved_tensors
        dl = opt_grad
        if ctx.padding == "valid":
            h = _get_halo(ctx.window_size)
            dl = torch.zeros_like(img1)
            dl[:, :, h:-h, h:-h] = opt_grad
        grad = ext.fusedssim_backward(ctx.window_size, ctx.C1, ctx.C2, img1, img2, dl, p0, p1, p2)
        return None, None, grad, None, None, None, None


class FusedSSIMMapFP16(torch.autograd.Function):
    """FP16-input SSIM map with FP32 arithmetic (reference: fussim/__init__.py:398-448).

    ``apply(C1, C2, img1, img2, padding="same", window_size=11)``: the images are rounded to
    FP16, the map and the partials are FP32, the gradient is FP32.
    """

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, C1, C2, img1, img2, padding="same", window_size=11):
        ext = _ensure_cuda_extension()
        a = img1 if img1.dtype == torch.float16 else img1.half()
        b = img2 if img2.dtype == torch.float16 else img2.half()
        ssim_map, p0, p1, p2 = ext.fusedssim_fp16_train(window_size, C1, C2, a, b)
        h = _get_halo(window_size)
        if padding == "valid":
            ssim_map = ssim_map[:, :, h:-h, h:-h]
        ctx.save_for_backward(a, b, p0, p1, p2)
        ctx.C1, ctx.C2, ctx.padding, ctx.window_size = C1, C2, padding, window_size
        return ssim_map

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, opt_grad):
        ext = _ensure_cuda_extension()
        a, b, p0, p1, p2 = ctx.saved_tensors
        dl = opt_grad.float()
        if ctx.padding == "valid":
            h = _get_halo(ctx.window_size)
            dl = torch.zeros(a.shape, dtype=torch.float32, device=a.device)
            dl[:, :, h:-h, h:-h] = opt_grad.float()
        grad = ext.fusedssim_fp16_backward(ctx.window_size, ctx.C1, ctx.C2, a, b, dl, p0, p1, p2)
        return None, None, grad, None, None, None


# ------------------------------------------------------------------------------------
# Fused loss: forward = partials + in-kernel reduction, backward = one kernel
# ------------------------------------------------------------------------------------
def _kernel_inputs(img1, img2, half):
    if half:
        a = img1 if img1.dtype == torch.float16 else img1.half()
        b = img2 if img2.dtype == torch.float16 else img2.half()
        return a, b
    return img1, (img2 if img2.dtype == img1.dtype else img2.to(img1.dtype))


def _reduce(img1, img2, C1, C2, window_size, valid, clamp, reduce, train, half):
    ext = _ensure_cuda_extension()
    if train:
        # autograd function implemented in the extension (C++): forward = fused kernel with
        # partials and in-kernel mean, backward = one kernel; d(out)/d(map) = 1/count, and
        # with nothing counted (an empty valid crop) no pixel receives gradient, as the
        # reference's zero-filled dL/dmap gives
        scale = _inv(_count(img1.shape, window_size, valid, reduce == _REDUCE_PER_IMAGE))
        chain = scale if scale != float("inf") else 0.0
        return ext.fused_loss(img1, img2, C1, C2, window_size, valid, clamp, reduce, half,
                              scale, chain, 0.0, 0.0, 0.0)
    a, b = _kernel_inputs(img1, img2, half)
    scale = _inv(_count(a.shape, window_size, valid, reduce == _REDUCE_PER_IMAGE))
    out, _, _ = ext.loss_forward(a, b, window_size, C1, C2, valid, clamp, False, reduce, False,
                                 scale)
    return out


def _float_path_inputs(img1, img2):
    # Outside autocast the reference's FP32 kernels take float32 tensors. Here half tensors
    # are read natively by the FP16-input kernels, a bfloat16 pair by the bfloat16-input
    # kernels (FP32 arithmetic and FP32 taps on the widened values: the same result as the
    # float32 path on img.float()), and a bfloat16 image paired with another dtype is
    # widened to float32.
    if (img1.dtype == torch.bfloat16) != (img2.dtype == torch.bfloat16):
        if img1.dtype == torch.bfloat16:
            img1 = img1.float()
        if img2.dtype == torch.bfloat16:
            img2 = img2.float()
    return img1, img2


def fused_ssim(
    img1: torch.Tensor,
    img2: torch.Tensor,
    padding: str = "same",
    train: bool = True,
    window_size: int = 11,
) -> torch.Tensor:
    """Mean SSIM of two (B, C, H, W) CUDA images; differentiable with respect to img1.

    Same contract as the reference (fussim/__init__.py:451-580): ``padding`` is "same"
    (zero padding) or "valid" (map cropped by (window_size-1)/2), ``window_size`` is one of
    7, 9, 11, ``train`` is honoured only when grad mode is on and img1 requires grad, and
    under ``torch.autocast`` the FP16 path runs. Returns a 0-d float32 tensor.
    """
    if not torch.cuda.is_available():
        raise RuntimeError(
            "CUDA is not available. fused_ssim requires a CUDA-capable GPU.\n"
            "If you have a GPU, make sure:\n"
            "  1. NVIDIA drivers are installed\n"
            "  2. PyTorch is installed with CUDA support"
        )
    if not img1.is_cuda:
        raise RuntimeError(
            f"img1 must be on a CUDA device, but got device: {img1.device}\n"
            "Move your tensor to GPU with: img1 = img1.cuda()"
        )
    if not img2.is_cuda:
        raise RuntimeError(
            f"img2 must be on a CUDA device, but got device: {img2.device}\n"
            "Move your tensor to GPU with: img2 = img2.cuda()"
        )
    if img1.device != img2.device:
        raise RuntimeError(
            "img1 and img2 must be on the same device.\n"
            f"img1 device: {img1.device}, img2 device: {img2.device}"
        )
    if img1.shape != img2.shape:
        raise ValueError(
            "img1 and img2 must have the same shape.\n"
            f"img1 shape: {img1.shape}, img2 shape: {img2.shape}"
        )
    if len(img1.shape) != 4:
        raise ValueError(
            f"Expected 4D tensor (B, C, H, W), but got {len(img1.shape)}D tensor "
            f"with shape {img1.shape}"
        )
    if padding not in ALLOWED_PADDING:
        raise ValueError(f"padding must be one of {ALLOWED_PADDING}, but got '{padding}'")
    if window_size not in SUPPORTED_WINDOW_SIZES:
        raise ValueError(f"window_size must be one of {SUPPORTED_WINDOW_SIZES}, got {window_size}")

    C1 = 0.01**2
    C2 = 0.03**2
    train = train and torch.is_grad_enabled() and img1.requires_grad
    half = torch.is_autocast_enabled()
    if not half:
        img1, img2 = _float_path_inputs(img1, img2)
    return _reduce(img1, img2, C1, C2, window_size, padding == "valid", False, _REDUCE_SCALAR,
                   train, half)


def l1_dssim_loss(
    img1: torch.Tensor,
    img2: torch.Tensor,
    lambda_dssim: float = 0.2,
    padding: str = "same",
    window_size: int = 11,
) -> torch.Tensor:
    """The 3D Gaussian Splatting photometric loss in one fused forward and one backward:

        (1 - lambda_dssim) * mean|img1 - img2| + lambda_dssim * (1 - fused_ssim(img1, img2))

    (the combination in the reference's tests/test_amp.py:223-227). The L1 mean runs over
    every pixel; the SSIM mean follows ``padding`` as in ``fused_ssim``. The forward kernel
    sums |img1 - img2| alongside the SSIM map and the backward kernel adds the L1 gradient
    (sign(img1 - img2) / N, 0 where equal), so neither image is read again for the L1 term.
    Differentiable with respect to img1; under autocast the FP16 path runs (the L1 term is
    then computed from the half-rounded images). Returns a 0-d float32 tensor.
    """
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available. l1_dssim_loss requires a CUDA-capable GPU.")
    if not img1.is_cuda or not img2.is_cuda:
        raise RuntimeError("img1 and img2 must be on a CUDA device")
    if img1.device != img2.device:
        raise RuntimeError("img1 and img2 must be on the same device.")
    if img1.shape != img2.shape:
        raise ValueError(
            "img1 and img2 must have the same shape.\n"
            f"img1 shape: {img1.shape}, img2 shape: {img2.shape}"
        )
    if len(img1.shape) != 4:
        raise ValueError(
            f"Expected 4D tensor (B, C, H, W), but got {len(img1.shape)}D tensor "
            f"with shape {img1.shape}"
        )
    if padding not in ALLOWED_PADDING:
        raise ValueError(f"padding must be one of {ALLOWED_PADDING}, but got '{padding}'")
    if window_size not in SUPPORTED_WINDOW_SIZES:
        raise ValueError(f"window_size must be one of {SUPPORTED_WINDOW_SIZES}, got {window_size}")
    lam = float(lambda_dssim)
    if not 0.0 <= lam <= 1.0:
        raise ValueError(f"lambda_dssim must be in [0, 1], got {lambda_dssim}")
    half = torch.is_autocast_enabled()
    if not half:
        img1, img2 = _float_path_inputs(img1, img2)
    valid = padding == "valid"
    ext = _ensure_cuda_extension()
    inv_ssim = _inv(_count(img1.shape, window_size, valid, False))
    inv_all = _inv(img1.numel())
    ssim_scale = -lam * inv_ssim if inv_ssim != float("inf") else 0.0
    l1_scale = (1.0 - lam) * inv_all if inv_all != float("inf") else 0.0
    if torch.is_grad_enabled() and img1.requires_grad:
        return ext.fused_loss(img1, img2, 0.01**2, 0.03**2, window_size, valid, False,
                              _REDUCE_SCALAR, half, ssim_scale, ssim_scale, l1_scale, lam,
                              l1_scale)
    a, b = _kernel_inputs(img1, img2, half)
    out, _, _ = ext.loss_forward(a, b, window_size, 0.01**2, 0.03**2, valid, False, False,
                                 _REDUCE_SCALAR, False, ssim_scale, l1_scale, lam)
    return out


def ssim(
    X: torch.Tensor,
    Y: torch.Tensor,
    data_range: float = 255,
    size_average: bool = True,
    win_size: int = 11,
    win_sigma: float = 1.5,
    win: torch.Tensor = None,
    K: tuple = (0.01, 0.03),
    nonnegative_ssim: bool = False,
) -> torch.Tensor:
    """pytorch-msssim compatible SSIM (reference: fussim/__init__.py:595-695).

    Always 'valid' padding; ``size_average=False`` returns shape (B,); ``nonnegative_ssim``
    clamps the per-pixel map at 0 (the reference's semantics) before reducing.
    """
    C1, C2 = _msssim_constants(data_range, win_size, win_sigma, win, K)
    train = torch.is_grad_enabled() and X.requires_grad
    half = torch.is_autocast_enabled()
    if not half:
        X, Y = _float_path_inputs(X, Y)
    reduce = _REDUCE_SCALAR if size_average else _REDUCE_PER_IMAGE
    return _reduce(X, Y, C1, C2, win_size, True, bool(nonnegative_ssim), reduce, train, half)


def _msssim_constants(data_range, win_size, win_sigma, win, K):
    """The pytorch-msssim argument checks of the reference's ``ssim`` (same messages, same
    order: fussim/__init__.py:636-658); returns (C1, C2)."""
    if win_size not in SUPPORTED_WINDOW_SIZES:
        raise ValueError(
            f"win_size must be one of {SUPPORTED_WINDOW_SIZES}, got {win_size}. "
            "These are the window sizes supported by the optimized CUDA kernels."
        )
    if win_sigma != 1.5:
        raise ValueError(
            f"win_sigma must be 1.5 (CUDA kernel limitation), got {win_sigma}. "
            "This is the standard SSIM sigma used by most implementations."
        )
    if win is not None:
        raise ValueError(
            "Custom window (win) is not supported. The CUDA kernel uses an "
            f"optimized built-in {win_size}x{win_size} Gaussian window with sigma=1.5."
        )
    if not (isinstance(K, (tuple, list)) and len(K) == 2):
        raise ValueError(f"K must be a tuple/list of 2 values (K1, K2), got {K}")
    K1, K2 = K
    if not (0 < K1 < 1 and 0 < K2 < 1):
        raise ValueError(f"K values must be in (0, 1), got K1={K1}, K2={K2}")
    return (K1 * data_range) ** 2, (K2 * data_range) ** 2


class SSIM(torch.nn.Module):
    """pytorch-msssim compatible module (reference: fussim/__init__.py:698-780)."""

    def __init__(
        self,
        data_range: float = 255,
        size_average: bool = True,
        win_size: int = 11,
        win_sigma: float = 1.5,
        channel: int = 3,
        spatial_dims: int = 2,
        K: tuple = (0.01, 0.03),
        nonnegative_ssim: bool = False,
    ):
        super().__init__()
        if win_size not in SUPPORTED_WINDOW_SIZES:
            raise ValueError(f"win_size must be one of {SUPPORTED_WINDOW_SIZES}, got {win_size}")
        if win_sigma != 1.5:
            raise ValueError(f"win_sigma must be 1.5 (CUDA kernel limitation), got {win_sigma}")
        if spatial_dims != 2:
            raise ValueError(f"spatial_dims must be 2 (only 2D images supported), got {spatial_dims}")
        if not (isinstance(K, (tuple, list)) and len(K) == 2):
            raise ValueError(f"K must be a tuple/list of 2 values (K1, K2), got {K}")
        if not (0 < K[0] < 1 and 0 < K[1] < 1):
            raise ValueError(f"K values must be in (0, 1), got K1={K[0]}, K2={K[1]}")
        self.data_range = data_range
        self.size_average = size_average
        self.win_size = win_size
        self.K = tuple(K)
        self.nonnegative_ssim = nonnegative_ssim
        # channel is accepted for compatibility and inferred from the input

    def forward(self, X: torch.Tensor, Y: torch.Tensor) -> torch.Tensor:
        return ssim(
            X,
            Y,
            data_range=self.data_range,
            size_average=self.size_average,
            win_size=self.win_size,
            K=self.K,
            nonnegative_ssim=self.nonnegative_ssim,
        )
