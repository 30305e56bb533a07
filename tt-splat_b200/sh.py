"""View-dependent colour from real spherical harmonics, degrees 0-3 (spike/sh.py:49-72), on the
device.

``eval_sh_color(deg, coeffs, dirs)`` keeps the reference's signature: coeffs [G, nc, 3] with
nc >= (deg+1)^2 (DC first, then the higher bands in the inria/gsplat order), dirs [G, 3]
(normalised inside, norm clamped at 1e-12); it returns clamp(0.5 + sum_k basis_k coeffs_k,
min 0) [G, 3].  A torch autograd Function over ``tts_eval_sh`` / ``tts_eval_sh_bwd`` (float32 or
float64) gives the gradients of the coefficients and of the directions; CPU tensors raise.

The basis constants below are the standard real-SH normalisations (the same numbers every 3DGS
code uses); the kernels carry their own copy.
"""
import torch

from . import ops
from ._lib import on_device

C0 = 0.28209479177387814
C1 = 0.4886025119029199
C2 = [1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792, 0.5462742152960396]
C3 = [-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154, -0.4570457994644658,
      1.445305721320277, -0.5900435899266435]


class _EvalSH(torch.autograd.Function):
    @staticmethod
    def forward(ctx, coeffs, dirs, deg):
        if coeffs.dim() < 2 or dirs.shape[-1] != 3 or coeffs.shape[:-2] != dirs.shape[:-1]:
            raise ValueError(f"coeffs [...,nc,3] and dirs [...,3] with the same leading dims, got "
                             f"{tuple(coeffs.shape)} and {tuple(dirs.shape)}")
        c, d = coeffs.detach().contiguous(), dirs.detach().contiguous()
        ctx.save_for_backward(c, d)
        ctx.deg = deg
        return ops.eval_sh(deg, c, d)

    @staticmethod
    def backward(ctx, gout):
        c, d = ctx.saved_tensors
        gco, gd = ops.eval_sh_bwd(ctx.deg, c, d, gout.contiguous())
        return gco, gd, None


def eval_sh_color(deg, coeffs, dirs):
    """spike/sh.py:49-72 on the device: RGB colour [..., 3] of SH degree ``deg`` (0..3)."""
    if int(deg) not in (0, 1, 2, 3):
        raise ValueError(f"SH degree must be 0..3, got {deg}")
    with on_device(coeffs):
        return _EvalSH.apply(coeffs, dirs, int(deg))
