"""The per-pixel forward primitives (mirrors spike/forward.py:13-71).

These small tensor expressions are the reference's building blocks and stay as torch
expressions on the caller's tensors; the hot path never calls them (the fused kernels evaluate
the same algebra per tile).  ``theta_from_conic`` and ``phi`` define the monomial map the
kernels implement: Q = Phi . theta with Phi = [px^2, py^2, px*py, px, py, 1].
"""
import torch

C0 = 0.28209479177387814


def quad_form(px, py, mu2d, conic_abc):
    """spike/forward.py:13-20: Q[P,G] raw Mahalanobis (no /k)."""
    dx = px[:, None] - mu2d[None, :, 0]
    dy = py[:, None] - mu2d[None, :, 1]
    a, b, c = conic_abc[:, 0][None, :], conic_abc[:, 1][None, :], conic_abc[:, 2][None, :]
    return a * dx * dx + 2 * b * dx * dy + c * dy * dy


def theta_from_conic(conic_abc, mu2d, k):
    """spike/forward.py:23-39: theta_Q[G,6], theta_u[G,6] (u = 1 - Q/k folded)."""
    a, b, c = conic_abc[:, 0], conic_abc[:, 1], conic_abc[:, 2]
    mux, muy = mu2d[:, 0], mu2d[:, 1]
    theta_Q = torch.stack([a, c, 2 * b, -2 * (a * mux + b * muy), -2 * (b * mux + c * muy),
                           a * mux * mux + 2 * b * mux * muy + c * muy * muy], dim=-1)
    bump = torch.zeros_like(theta_Q)
    bump[..., 5] = 1.0
    return theta_Q, (-1.0 / k) * theta_Q + bump


def phi(px, py):
    """spike/forward.py:42-44."""
    return torch.stack([px * px, py * py, px * py, px, py, torch.ones_like(px)], dim=-1)


def quad_form_tilelocal(lx, ly, conic_abc, mu2d, tile_origin):
    """spike/forward.py:47-58: tile-local exact GEMM form of Q."""
    theta_Q, _ = theta_from_conic(conic_abc, mu2d - tile_origin, k=1.0)
    return phi(lx, ly) @ theta_Q.transpose(-1, -2)


def poly_splat_wgeo(Q, k, keep=None):
    """spike/forward.py:61-66: max(0, 1 - Q/k)^2, keep-gated."""
    w_geo = (1.0 - Q / k).clamp(min=0.0) ** 2
    if keep is not None:
        w_geo = w_geo * keep[None, :].to(w_geo.dtype)
    return w_geo


def color_from_dc(color_dc):
    """spike/forward.py:69-71."""
    return (0.5 + C0 * color_dc).clamp(min=0.0)
