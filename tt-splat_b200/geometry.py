"""Gaussian geometry on the device: the differentiable functions of spike/geometry.py:10-57.

``quat_to_rotmat(quats)``, ``cov3d(scales, R)`` and ``project_ewa(means3d, cov3d_w, R_v, t_v,
fx, fy, cx, cy, blur_eps, near)`` keep the reference's signatures, shapes and clamps (quaternion
norm and 2-D determinant at 1e-12, depth at ``near``).  Each is a torch autograd Function whose
forward and backward are kernels of ``libttsplat_b200.so`` (``tts_quat_to_rotmat``,
``tts_cov3d``, ``tts_project_ewa`` and their ``_bwd``), in float32 or float64; CPU tensors raise
(there is no CPU fallback).  The camera (R_v, t_v and the intrinsics) is a constant: it receives
no gradient, as in every training path of the reference.

``project(model, cams)`` is the fused path the renderer and the train step use: geometry, SH
colour and activations of every gaussian in every view in one kernel.
"""
import torch

from . import ops
from ._lib import on_device
from .camera import as_camera, pack_cameras
from .model import flat_of


def _lead(x, tail, name):
    if x.dim() < len(tail) or tuple(x.shape[x.dim() - len(tail):]) != tail:
        raise ValueError(f"{name} must end in {tail}, got {tuple(x.shape)}")
    return x.contiguous()


class _QuatToRotmat(torch.autograd.Function):
    @staticmethod
    def forward(ctx, quats):
        q = _lead(quats.detach(), (4,), "quats")
        ctx.save_for_backward(q)
        return ops.quat_to_rotmat(q)

    @staticmethod
    def backward(ctx, gR):
        (q,) = ctx.saved_tensors
        return ops.quat_to_rotmat_bwd(q, gR.contiguous())


class _Cov3d(torch.autograd.Function):
    @staticmethod
    def forward(ctx, scales, R):
        s = _lead(scales.detach(), (3,), "scales")
        r = _lead(R.detach(), (3, 3), "R")
        if s.shape[:-1] != r.shape[:-2]:
            raise ValueError(f"scales {tuple(s.shape)} and R {tuple(r.shape)} must share their leading dims")
        ctx.save_for_backward(s, r)
        return ops.cov3d(s, r)

    @staticmethod
    def backward(ctx, gcov):
        s, r = ctx.saved_tensors
        return ops.cov3d_bwd(s, r, gcov.contiguous())


class _ProjectEwa(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means3d, cov3d_w, cam16, blur, near):
        m = _lead(means3d.detach(), (3,), "means3d")
        c = _lead(cov3d_w.detach(), (3, 3), "cov3d_w")
        if m.dim() != 2 or c.shape[0] != m.shape[0]:
            raise ValueError("project_ewa takes means3d [G,3] and cov3d_w [G,3,3]")
        mu2d, conic, depth, keep = ops.project_ewa(m, c, cam16, blur, near)
        ctx.save_for_backward(m, c)
        ctx.args = (cam16, blur, near)
        ctx.mark_non_differentiable(keep)
        return mu2d, conic, depth, keep

    @staticmethod
    def backward(ctx, gmu2d, gconic, gdepth, _gkeep):
        m, c = ctx.saved_tensors
        cam16, blur, near = ctx.args
        f = lambda g: None if g is None else g.contiguous()  # noqa: E731
        gm, gc = ops.project_ewa_bwd(m, c, cam16, blur, near, f(gmu2d), f(gconic), f(gdepth))
        return gm, gc, None, None, None


def quat_to_rotmat(quats):
    """quats [...,4] (w, x, y, z; normalised, norm clamped at 1e-12) -> R [...,3,3]
    (spike/geometry.py:10-19)."""
    with on_device(quats):
        return _QuatToRotmat.apply(quats)


def cov3d(scales, R):
    """R diag(scales^2) R^T for scales [...,3] (already exponentiated) and R [...,3,3]
    (spike/geometry.py:22-25)."""
    with on_device(scales):
        return _Cov3d.apply(scales, R)


def project_ewa(means3d, cov3d_w, R_v, t_v, fx, fy, cx, cy, blur_eps=0.3, near=0.2):
    """EWA projection (spike/geometry.py:28-57) -> mu2d [G,2], conic_abc [G,3], depth [G],
    keep [G] (bool).  Differentiable in means3d and cov3d_w."""
    cam16 = ops._cam16(R_v, t_v, fx, fy, cx, cy)
    with on_device(means3d):
        return _ProjectEwa.apply(means3d, cov3d_w, cam16, float(blur_eps), float(near))


@torch.no_grad()
def project(model, cams, sh_degree=0, blur_eps=0.3, near=0.2):
    """Fused projection of every gaussian into every view (device kernel):
    returns dict(mu2d[V,G,2], conic[V,G,3], color_o[V,G,3], keo[V,G], depth[V,G], keep[V,G])."""
    cams = [as_camera(c) for c in cams]
    flat = flat_of(model).detach().contiguous()
    G = model.means3d.shape[0]
    pj = ops.project(flat, G, sh_degree, pack_cameras(cams, flat.device), cams[0].H, cams[0].W, blur_eps, near)
    p = pj["proj"]
    return dict(mu2d=pj["mu2d"], conic=p[..., 2:5], color_o=p[..., 5:8], keo=p[..., 8], depth=p[..., 9],
                keep=pj["keep"].bool())
