"""fussim_b200 — differentiable SSIM for PyTorch on NVIDIA B200 (sm_100a).

Drop-in for the public API of OpsiClear/fussim (``fussim/__init__.py``):

* ``fused_ssim(img1, img2, padding="same", train=True, window_size=11)`` — scalar mean SSIM;
* ``ssim`` / ``SSIM`` — the pytorch-msssim compatible wrappers (``size_average=False``
  returns one value per image);
* ``FusedSSIMMap`` / ``FusedSSIMMapFP16`` — the map-producing autograd Functions;
* ``SUPPORTED_WINDOW_SIZES``, ``get_build_info``, ``check_compatibility``.

Gradients flow to the first image only. Under ``torch.autocast`` the inputs are rounded
to FP16 (whatever the autocast dtype, as the reference does) and the arithmetic stays
FP32. There is no CPU path: every call runs the hand-written sm_100a kernels of
``libfussim_b200.so`` and fails loudly if they are missing.
"""

from .functional import (  # noqa: F401
    ALLOWED_PADDING,
    SSIM,
    SUPPORTED_WINDOW_SIZES,
    FusedSSIMMap,
    FusedSSIMMapFP16,
    __version__,
    check_compatibility,
    check_device_errors,
    fused_ssim,
    get_build_info,
    l1_dssim_loss,
    poll_device_error,
    ssim,
)

__all__ = [
    # Primary API
    "fused_ssim",
    "l1_dssim_loss",
    # pytorch-msssim compatible API
    "ssim",
    "SSIM",
    # Advanced/internal
    "FusedSSIMMap",
    "FusedSSIMMapFP16",
    # Utilities
    "__version__",
    "get_build_info",
    "check_compatibility",
    "check_device_errors",
    "poll_device_error",
    "SUPPORTED_WINDOW_SIZES",
]
