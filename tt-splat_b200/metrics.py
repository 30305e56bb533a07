"""Image metrics and the photometric loss (mirrors spike/metrics.py:1-28).

``loss_fn`` runs the fused L1 + SSIM kernel, which returns the loss and its gradient in one
pass; the autograd backward scales the stored gradient.  Images are [H,W,3] (or [V,H,W,3]).
"""
import torch

from ._lib import on_device
from . import ops


class _LossFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, gt, lam):
        p = pred.detach().float().contiguous()
        g = gt.detach().float().contiguous().to(p.device)
        out = ops.loss_l1_ssim(p, g, lam, 1.0)
        ctx.save_for_backward(out["gimg"].reshape(pred.shape))
        return out["loss"].sum()

    @staticmethod
    def backward(ctx, gout):
        (gimg,) = ctx.saved_tensors
        return gimg * gout, None, None


def loss_fn(pred, gt, lambda_ssim=0.2):
    """(1-l)*L1 + l*(1-SSIM) (spike/metrics.py:26-28); SSIM on [0,1]-clamped inputs, window 11
    shrunk for small images (:15-19).  For a [V,H,W,3] batch, the sum of the per-view losses."""
    with on_device(pred):
        return _LossFn.apply(pred, gt, float(lambda_ssim))


def psnr(pred, gt):
    """spike/metrics.py:10-12."""
    mse = (pred.clamp(0.0, 1.0) - gt.clamp(0.0, 1.0)).pow(2).mean()
    return -10.0 * torch.log10(mse.clamp(min=1e-12))


def l1(pred, gt):
    """spike/metrics.py:22-23."""
    return (pred - gt).abs().mean()


def ssim(pred, gt, win_size=11):
    """SSIM of [H,W,3] images (spike/metrics.py:15-19) from the fused kernel (lambda = 1 makes
    the loss 1 - SSIM)."""
    return 1.0 - ops.loss_l1_ssim(pred.detach().float().contiguous(), gt.float().contiguous().to(pred.device),
                                  1.0, 1.0)["loss"].sum()
