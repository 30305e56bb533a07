"""Gaussian geometry (mirrors spike/geometry.py:10-57).

``project(model, cams)`` is the B200 path: the fused projection kernel (geometry + SH colour +
activations) for a batch of views.  ``quat_to_rotmat``, ``cov3d`` and ``project_ewa`` keep the
reference's tensor expressions for callers that compose them by hand.
"""
import torch

from . import ops
from .camera import as_camera, pack_cameras
from .model import flat_of


def quat_to_rotmat(quats):
    """spike/geometry.py:10-19."""
    q = quats / quats.norm(dim=-1, keepdim=True).clamp(min=1e-12)
    w, x, y, z = q[..., 0], q[..., 1], q[..., 2], q[..., 3]
    return torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
                        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
                        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)],
                       dim=-1).reshape(*q.shape[:-1], 3, 3)


def cov3d(scales, R):
    """spike/geometry.py:22-25."""
    s2 = scales * scales
    return (R * s2[..., None, :]) @ R.transpose(-1, -2)


def project_ewa(means3d, cov3d_w, R_v, t_v, fx, fy, cx, cy, blur_eps=0.3, near=0.2):
    """spike/geometry.py:28-57."""
    mu_cam = means3d @ R_v.transpose(-1, -2) + t_v
    depth = mu_cam[:, 2]
    keep = depth > near
    z = depth.clamp(min=near)
    mu2d = torch.stack([fx * mu_cam[:, 0] / z + cx, fy * mu_cam[:, 1] / z + cy], dim=-1)
    Sigma_cam = torch.einsum('ij,gjk,lk->gil', R_v, cov3d_w, R_v)
    zero = torch.zeros_like(z)
    J = torch.stack([torch.stack([fx / z, zero, -fx * mu_cam[:, 0] / (z * z)], dim=-1),
                     torch.stack([zero, fy / z, -fy * mu_cam[:, 1] / (z * z)], dim=-1)], dim=-2)
    Sigma2d = torch.einsum('gij,gjk,glk->gil', J, Sigma_cam, J) + blur_eps * torch.eye(2, dtype=J.dtype, device=J.device)
    s00, s01, s11 = Sigma2d[:, 0, 0], Sigma2d[:, 0, 1], Sigma2d[:, 1, 1]
    det = (s00 * s11 - s01 * s01).clamp(min=1e-12)
    return mu2d, torch.stack([s11 / det, -s01 / det, s00 / det], dim=-1), depth, keep


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
