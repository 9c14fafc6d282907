"""Seeded synthetic image pairs for the SSIM workloads.

All generators draw from a CPU ``torch.Generator`` so that the same seed produces the
same bytes on every machine; callers move the result to the device themselves.

Workloads (B, C, H, W; value distributions):

* ``pair_noise``    img1 ~ U[0,1], img2 = clamp(img1 + N(0, sigma^2), 0, 1)
  (the 1x3x256^2 unit case with sigma=0.05, the 64x3x2048^2 batch sweep with sigma=0.1).
* ``pair_blobs``    img2 = sum of 200 anisotropic Gaussian blobs (random centres, sigma
  5-80 px, random orientation, RGB amplitudes U[0,1]) normalised to [0,1]; img1 =
  clamp(box3x3(img2) + N(0, 0.03^2), 0, 1). The 3DGS-like render/ground-truth pair used
  for the 1080p RGB step and the 8x3x1024^2 FP16 case.
* ``pair_uniform``  independent U[0,1] pairs (the 3x1x517x999 edge case).
"""

from __future__ import annotations

import math

import torch


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    return g


def pair_uniform(shape, seed: int = 0, dtype=torch.float32):
    g = _gen(seed)
    a = torch.rand(shape, generator=g, dtype=torch.float32)
    b = torch.rand(shape, generator=g, dtype=torch.float32)
    return a.to(dtype), b.to(dtype)


def pair_noise(shape, sigma: float, seed: int = 0, dtype=torch.float32):
    g = _gen(seed)
    a = torch.rand(shape, generator=g, dtype=torch.float32)
    b = (a + sigma * torch.randn(shape, generator=g, dtype=torch.float32)).clamp_(0.0, 1.0)
    return a.to(dtype), b.to(dtype)


def blob_field(channels: int, height: int, width: int, g: torch.Generator, n_blobs: int = 200):
    """Sum of ``n_blobs`` anisotropic Gaussian blobs, normalised to [0, 1]. Shape (C, H, W)."""
    cy = torch.rand(n_blobs, generator=g, dtype=torch.float64) * height
    cx = torch.rand(n_blobs, generator=g, dtype=torch.float64) * width
    sa = 5.0 + 75.0 * torch.rand(n_blobs, generator=g, dtype=torch.float64)
    sb = 5.0 + 75.0 * torch.rand(n_blobs, generator=g, dtype=torch.float64)
    th = math.pi * torch.rand(n_blobs, generator=g, dtype=torch.float64)
    amp = torch.rand(n_blobs, channels, generator=g, dtype=torch.float64)
    ys = torch.arange(height, dtype=torch.float32).view(height, 1)
    xs = torch.arange(width, dtype=torch.float32).view(1, width)
    field = torch.zeros(channels, height, width, dtype=torch.float32)
    for i in range(n_blobs):
        c, s = math.cos(th[i].item()), math.sin(th[i].item())
        a2, b2 = 2.0 * sa[i].item() ** 2, 2.0 * sb[i].item() ** 2
        # only evaluate inside a 4-sigma bounding box: the blob is ~0 outside
        r = 4.0 * max(sa[i].item(), sb[i].item())
        y0, y1 = max(0, int(cy[i] - r)), min(height, int(cy[i] + r) + 1)
        x0, x1 = max(0, int(cx[i] - r)), min(width, int(cx[i] + r) + 1)
        if y0 >= y1 or x0 >= x1:
            continue
        dy = ys[y0:y1] - float(cy[i])
        dx = xs[:, x0:x1] - float(cx[i])
        u = c * dx + s * dy
        v = -s * dx + c * dy
        e = torch.exp(-(u * u) / a2 - (v * v) / b2)
        field[:, y0:y1, x0:x1] += amp[i].to(torch.float32).view(channels, 1, 1) * e
    lo, hi = field.min(), field.max()
    return (field - lo) / (hi - lo + 1e-12)


def box3x3(x: torch.Tensor) -> torch.Tensor:
    """3x3 mean filter with zero padding, per channel. x: (B, C, H, W)."""
    c = x.shape[1]
    k = torch.full((c, 1, 3, 3), 1.0 / 9.0, dtype=x.dtype)
    return torch.nn.functional.conv2d(x, k, padding=1, groups=c)


def pair_blobs(shape, seed: int = 0, dtype=torch.float32, noise: float = 0.03):
    """(render-like img1, ground-truth-like img2) pair, see module docstring."""
    b, c, h, w = shape
    g = _gen(seed)
    gt = torch.stack([blob_field(c, h, w, g) for _ in range(b)])
    render = box3x3(gt) + noise * torch.randn(gt.shape, generator=g, dtype=torch.float32)
    render.clamp_(0.0, 1.0)
    return render.to(dtype).contiguous(), gt.to(dtype).contiguous()


# Named workloads (shape, generator) used by the benchmark and the tests.
WORKLOADS = {
    "unit_256": dict(shape=(1, 3, 256, 256), kind="noise", sigma=0.05, dtype=torch.float32,
                     padding="same", window=11),
    "rgb_1080p": dict(shape=(1, 3, 1080, 1920), kind="blobs", dtype=torch.float32,
                      padding="same", window=11),
    "fp16_1024_valid": dict(shape=(8, 3, 1024, 1024), kind="blobs", dtype=torch.float16,
                            padding="valid", window=11),
    "batch_2048": dict(shape=(64, 3, 2048, 2048), kind="noise", sigma=0.1, dtype=torch.float32,
                       padding="same", window=11),
    "edge_517x999": dict(shape=(3, 1, 517, 999), kind="uniform", dtype=torch.float32,
                         padding="same", window=11),
}


def make_pair(name: str, seed: int = 0, shape=None):
    """Generate the named workload's pair on the CPU (optionally with another shape)."""
    spec = WORKLOADS[name]
    shp = tuple(shape) if shape is not None else spec["shape"]
    if spec["kind"] == "noise":
        return pair_noise(shp, spec["sigma"], seed, spec["dtype"])
    if spec["kind"] == "blobs":
        return pair_blobs(shp, seed, spec["dtype"])
    return pair_uniform(shp, seed, spec["dtype"])
