"""The hand-derived WSR + poly-splat backward as an autograd Function (mirrors
spike/backward.py:11-63) on the dense CUDA kernels.

``wsr_polysplat(theta_u[G,6], o[G], color[G,3], w_b, Phi[P,6], c_b[3], keep[G]) -> C[P,3]``,
differentiable in theta_u, o, color and w_b like ``WSRPolySplatHot``.
"""
import torch

from ._lib import on_device
from . import ops


class WSRPolySplatHot(torch.autograd.Function):
    """Manual forward + backward on the CUDA kernels (spike/backward.py:23-58)."""

    @staticmethod
    def forward(ctx, theta_u, o, color, w_b, Phi, c_b, keep):
        f = lambda t: None if t is None else t.detach().float().contiguous()  # noqa: E731
        th, oo, col, Ph, cb, kp = f(theta_u), f(o), f(color), f(Phi), f(c_b), f(keep)
        wb = torch.as_tensor(w_b, dtype=torch.float32, device=th.device).detach().reshape(1).contiguous()
        C, den = ops.wsr_dense_fwd(th, oo, col, wb, Ph, cb, kp)
        ctx.save_for_backward(th, oo, col, wb, Ph, cb, C, den)
        ctx.keep = kp
        ctx.wb_shape = torch.as_tensor(w_b).shape
        return C

    @staticmethod
    def backward(ctx, gC):
        th, oo, col, wb, Ph, cb, C, den = ctx.saved_tensors
        gth, go, gcol, gwb = ops.wsr_dense_bwd(th, oo, col, wb, Ph, cb, ctx.keep, C, den, gC.float().contiguous())
        return gth, go, gcol, gwb.reshape(ctx.wb_shape), None, None, None


def wsr_polysplat(theta_u, o, color, w_b, Phi, c_b, keep=None):
    """spike/backward.py:61-63."""
    with on_device(theta_u):
        return WSRPolySplatHot.apply(theta_u, o, color, w_b, Phi, c_b, keep)
