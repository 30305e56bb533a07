"""Oracle: real spherical-harmonics colour, degrees 0-3, forward and manual backward.

Restates ``spike/sh.py:49-72`` (eval_sh_color): colour = clamp(0.5 + sum_k basis_k(d) c_k, min 0)
with d = dirs / clamp(|dirs|, 1e-12).  The backward is what torch autograd computes for that
expression (the reference's CPU path differentiates it with autograd, ``spike/render.py:22-25``):
coefficient grads basis_k * g * [0.5 + r >= 0] (torch's clamp passes the gradient at the bound)
and direction grads through the normalisation.  float64.
"""
import numpy as np

C0 = 0.28209479177387814                                   # spike/sh.py:9
C1 = 0.4886025119029199                                    # spike/sh.py:10
C2 = [1.0925484305920792, -1.0925484305920792, 0.31539156525252005,
      -1.0925484305920792, 0.5462742152960396]             # spike/sh.py:11-17
C3 = [-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154,
      -0.4570457994644658, 1.445305721320277, -0.5900435899266435]   # spike/sh.py:38-46


def _unit(dirs):
    dirs = np.asarray(dirs, np.float64)
    nrm = np.linalg.norm(dirs, axis=-1, keepdims=True)
    return dirs / np.maximum(nrm, 1e-12), nrm


def basis(deg, d):
    """[..., (deg+1)^2] basis values in the coefficient order of spike/sh.py:57-71."""
    x, y, z = d[..., 0], d[..., 1], d[..., 2]
    b = [np.full_like(x, C0)]
    if deg >= 1:
        b += [-C1 * y, C1 * z, -C1 * x]
    if deg >= 2:
        xx, yy, zz, xy, yz, xz = x * x, y * y, z * z, x * y, y * z, x * z
        b += [C2[0] * xy, C2[1] * yz, C2[2] * (2.0 * zz - xx - yy), C2[3] * xz, C2[4] * (xx - yy)]
    if deg >= 3:
        b += [C3[0] * y * (3 * xx - yy), C3[1] * xy * z, C3[2] * y * (4 * zz - xx - yy),
              C3[3] * z * (2 * zz - 3 * xx - 3 * yy), C3[4] * x * (4 * zz - xx - yy),
              C3[5] * z * (xx - yy), C3[6] * x * (xx - 3 * yy)]
    return np.stack(b, -1)


def basis_grad(deg, d):
    """d basis_k / d(x,y,z) -> [..., (deg+1)^2, 3] (derivatives of the polynomials above)."""
    x, y, z = d[..., 0], d[..., 1], d[..., 2]
    zero = np.zeros_like(x)
    rows = [(zero, zero, zero)]
    if deg >= 1:
        rows += [(zero, zero - C1, zero), (zero, zero, zero + C1), (zero - C1, zero, zero)]
    if deg >= 2:
        rows += [(C2[0] * y, C2[0] * x, zero), (zero, C2[1] * z, C2[1] * y),
                 (-2 * C2[2] * x, -2 * C2[2] * y, 4 * C2[2] * z), (C2[3] * z, zero, C2[3] * x),
                 (2 * C2[4] * x, -2 * C2[4] * y, zero)]
    if deg >= 3:
        xx, yy, zz = x * x, y * y, z * z
        rows += [(6 * C3[0] * x * y, C3[0] * (3 * xx - 3 * yy), zero),
                 (C3[1] * y * z, C3[1] * x * z, C3[1] * x * y),
                 (-2 * C3[2] * x * y, C3[2] * (4 * zz - xx - 3 * yy), 8 * C3[2] * y * z),
                 (-6 * C3[3] * x * z, -6 * C3[3] * y * z, C3[3] * (6 * zz - 3 * xx - 3 * yy)),
                 (C3[4] * (4 * zz - 3 * xx - yy), -2 * C3[4] * x * y, 8 * C3[4] * x * z),
                 (2 * C3[5] * x * z, -2 * C3[5] * y * z, C3[5] * (xx - yy)),
                 (C3[6] * (3 * xx - 3 * yy), -6 * C3[6] * x * y, zero)]
    return np.stack([np.stack(r, -1) for r in rows], -2)


def eval_sh_color(deg, coeffs, dirs):
    """spike/sh.py:49-72.  coeffs[G,(>=deg+1)^2,3], dirs[G,3] -> colour[G,3], pre-clamp r+0.5."""
    d, _ = _unit(dirs)
    nb = (deg + 1) ** 2
    B = basis(deg, d)
    pre = np.einsum("gk,gkc->gc", B, np.asarray(coeffs, np.float64)[:, :nb]) + 0.5
    return np.maximum(pre, 0.0), pre


def eval_sh_color_bwd(deg, coeffs, dirs, gcolor):
    """Autograd of eval_sh_color: (gcoeffs[G,(deg+1)^2,3], gdirs[G,3])."""
    d, nrm = _unit(dirs)
    nb = (deg + 1) ** 2
    _, pre = eval_sh_color(deg, coeffs, dirs)
    gr = np.asarray(gcolor, np.float64) * (pre >= 0.0)
    B = basis(deg, d)
    gco = B[:, :, None] * gr[:, None, :]
    dB = basis_grad(deg, d)                                             # [G,nb,3]
    gd = np.einsum("gkc,gkj,gc->gj", np.asarray(coeffs, np.float64)[:, :nb], dB, gr)
    big = nrm[:, 0] > 1e-12
    gdirs = np.where(big[:, None],
                     (gd - d * np.sum(d * gd, -1, keepdims=True)) / np.maximum(nrm, 1e-12),
                     gd / 1e-12)
    return gco, gdirs
