"""The reference's Python call sequence over the reference's own CUDA kernels.

Test infrastructure: restates what ``fussim/__init__.py`` of OpsiClear/fussim does around
its extension (``FusedSSIMMap`` :351-395, ``FusedSSIMMapFP16`` :398-448, ``fused_ssim``
:551-580, ``ssim`` :661-695) so parity tests can compare whole results — values and
gradients — with the engine under test on identical inputs.
"""

import torch

C1 = 0.01**2
C2 = 0.03**2


def _halo(ws):
    return (ws - 1) // 2


class RefMap(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ext, img1, img2, C1_, C2_, padding, window_size, fp16):
        if fp16:
            a = img1 if img1.dtype == torch.float16 else img1.half()
            b = img2 if img2.dtype == torch.float16 else img2.half()
            m, p0, p1, p2 = ext.fusedssim_fp16_train(window_size, C1_, C2_, a, b)
        else:
            a, b = img1, img2
            m, p0, p1, p2 = ext.fusedssim(window_size, C1_, C2_, a, b, True)
        h = _halo(window_size)
        if padding == "valid":
            m = m[:, :, h:-h, h:-h]
        ctx.save_for_backward(a, b, p0, p1, p2)
        ctx.cfg = (ext, C1_, C2_, padding, window_size, fp16)
        return m

    @staticmethod
    def backward(ctx, g):
        ext, C1_, C2_, padding, ws, fp16 = ctx.cfg
        a, b, p0, p1, p2 = ctx.saved_tensors
        dl = g.float()
        if padding == "valid":
            h = _halo(ws)
            dl = torch.zeros(a.shape, dtype=torch.float32, device=a.device)
            dl[:, :, h:-h, h:-h] = g.float()
        if fp16:
            grad = ext.fusedssim_fp16_backward(ws, C1_, C2_, a, b, dl, p0, p1, p2)
        else:
            grad = ext.fusedssim_backward(ws, C1_, C2_, a, b, dl, p0, p1, p2)
        return None, grad, None, None, None, None, None, None


def reference_loss(ext, img1, img2, window_size=11, padding="same", fp16=False, C1_=C1, C2_=C2,
                   clamp=False, per_image=False):
    m = RefMap.apply(ext, img1, img2, C1_, C2_, padding, window_size, fp16)
    if clamp:
        m = torch.clamp(m, min=0)
    return m.mean(dim=(1, 2, 3)) if per_image else m.mean()


def value_and_grad(fn, img1, img2, upstream=None):
    """Run fn(x, img2) on a fresh leaf copy of img1; return (value, grad of sum(up*value))."""
    x = img1.detach().clone().requires_grad_(True)
    v = fn(x, img2)
    up = torch.ones_like(v) if upstream is None else upstream
    (v * up).sum().backward()
    return v.detach(), x.grad.detach()
