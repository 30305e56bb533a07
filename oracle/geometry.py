"""Oracle: quaternion/scale -> 3D covariance -> EWA 2D conic, forward and manual backward.

Restates ``spike/geometry.py:10-57`` (quat_to_rotmat, cov3d, project_ewa) in the per-component
form of the reference's own manual geometry ``tools/geom_bwd.py:26-64`` (fwd) and
``tools/geom_bwd.py:67-152`` (bwd).  Evaluated in float64 (the reference's tests lock geometry
in fp64, ``spike/geometry.py:4-5``); outputs are cast to float32 by the callers that need the
fp32 pipeline values.
"""
import numpy as np

NEAR, BLUR = 0.2, 0.3          # tools/geom_bwd.py:23


def quat_to_rotmat(quats):
    """spike/geometry.py:10-19: normalised (clamp 1e-12) w,x,y,z quaternion -> R[...,3,3]."""
    q = np.asarray(quats, np.float64)
    n = np.maximum(np.linalg.norm(q, axis=-1, keepdims=True), 1e-12)
    w, x, y, z = np.moveaxis(q / n, -1, 0)
    R = np.stack([
        1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1)
    return R.reshape(q.shape[:-1] + (3, 3))


def cov3d(scales, R):
    """spike/geometry.py:22-25: R diag(s^2) R^T."""
    s2 = np.asarray(scales, np.float64) ** 2
    return (R * s2[..., None, :]) @ np.swapaxes(R, -1, -2)


def project_ewa(means3d, cov3d_w, R_v, t_v, fx, fy, cx, cy, blur_eps=BLUR, near=NEAR):
    """spike/geometry.py:28-57 (dense matrix form): mu2d[G,2], conic[G,3], depth[G], keep[G]."""
    m = np.asarray(means3d, np.float64)
    Rv = np.asarray(R_v, np.float64)
    mu_cam = m @ Rv.T + np.asarray(t_v, np.float64)
    depth = mu_cam[:, 2]
    keep = depth > near
    z = np.maximum(depth, near)
    mu2d = np.stack([fx * mu_cam[:, 0] / z + cx, fy * mu_cam[:, 1] / z + cy], -1)
    Sc = np.einsum("ij,gjk,lk->gil", Rv, np.asarray(cov3d_w, np.float64), Rv)
    zero = np.zeros_like(z)
    J = np.stack([np.stack([fx / z, zero, -fx * mu_cam[:, 0] / (z * z)], -1),
                  np.stack([zero, fy / z, -fy * mu_cam[:, 1] / (z * z)], -1)], -2)
    S2 = np.einsum("gij,gjk,glk->gil", J, Sc, J) + blur_eps * np.eye(2)
    s00, s01, s11 = S2[:, 0, 0], S2[:, 0, 1], S2[:, 1, 1]
    det = np.maximum(s00 * s11 - s01 * s01, 1e-12)
    conic = np.stack([s11 / det, -s01 / det, s00 / det], -1)
    return mu2d, conic, depth, keep


def fwd(means, quats, log_scales, cam, blur=BLUR, near=NEAR):
    """tools/geom_bwd.py:26-64 with scale = exp(log_scales); returns conic, mu2d, depth, keep
    and the cache the manual backward needs."""
    means = np.asarray(means, np.float64)
    quat = np.asarray(quats, np.float64)
    scale = np.exp(np.asarray(log_scales, np.float64))
    Rv = np.asarray(cam["R_v"], np.float64)
    tv = np.asarray(cam["t_v"], np.float64)
    fx, fy, cx, cy = (float(cam[k]) for k in ("fx", "fy", "cx", "cy"))
    mx, my, mz = means.T
    qw, qx, qy, qz = quat.T
    sx, sy, sz = scale.T
    n = np.maximum(np.sqrt(qw * qw + qx * qx + qy * qy + qz * qz), 1e-12)
    w, x, y, z = qw / n, qx / n, qy / n, qz / n
    R = [[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
         [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
         [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]]
    M = [[Rv[i][0] * R[0][k] + Rv[i][1] * R[1][k] + Rv[i][2] * R[2][k] for k in range(3)]
         for i in range(3)]
    s2 = [sx * sx, sy * sy, sz * sz]

    def SC(i, l):
        return M[i][0] * M[l][0] * s2[0] + M[i][1] * M[l][1] * s2[1] + M[i][2] * M[l][2] * s2[2]

    SC00, SC01, SC02, SC11, SC12, SC22 = SC(0, 0), SC(0, 1), SC(0, 2), SC(1, 1), SC(1, 2), SC(2, 2)
    mcx = Rv[0][0] * mx + Rv[0][1] * my + Rv[0][2] * mz + tv[0]
    mcy = Rv[1][0] * mx + Rv[1][1] * my + Rv[1][2] * mz + tv[1]
    mcz = Rv[2][0] * mx + Rv[2][1] * my + Rv[2][2] * mz + tv[2]
    zmask = (mcz > near).astype(np.float64)
    z_ = np.maximum(mcz, near)
    zi = 1.0 / z_
    mu2d = np.stack([fx * mcx * zi + cx, fy * mcy * zi + cy], -1)
    J00, J11 = fx * zi, fy * zi
    J02, J12 = -fx * mcx * zi * zi, -fy * mcy * zi * zi
    s00 = J00 * J00 * SC00 + 2 * J00 * J02 * SC02 + J02 * J02 * SC22 + blur
    s11 = J11 * J11 * SC11 + 2 * J11 * J12 * SC12 + J12 * J12 * SC22 + blur
    s01 = J00 * J11 * SC01 + J00 * J12 * SC02 + J02 * J11 * SC12 + J02 * J12 * SC22
    det = s00 * s11 - s01 * s01
    dmask = (det > 1e-12).astype(np.float64)
    deti = 1.0 / np.maximum(det, 1e-12)
    conic = np.stack([s11 * deti, -s01 * deti, s00 * deti], -1)
    cache = dict(w=w, x=x, y=y, z=z, n=n, M=M, s2=s2, sx=sx, sy=sy, sz=sz,
                 SC=[[SC00, SC01, SC02], [SC01, SC11, SC12], [SC02, SC12, SC22]],
                 mcx=mcx, mcy=mcy, zmask=zmask, zi=zi, J00=J00, J02=J02, J11=J11, J12=J12,
                 s00=s00, s11=s11, s01=s01, dmask=dmask, deti=deti, Rv=Rv, fx=fx, fy=fy,
                 scale=scale)
    return conic, mu2d, mcz, mcz > near, cache


def bwd(c, ga, gb, gc, gmux, gmuy):
    """tools/geom_bwd.py:67-152: (gconic, gmu2d) -> (gmeans[G,3], gquats[G,4], gscales[G,3])."""
    deti, s00, s11, s01 = c["deti"], c["s00"], c["s11"], c["s01"]
    gs11 = ga * deti
    gs01 = -gb * deti
    gs00 = gc * deti
    gdeti = ga * s11 + (-gb) * s01 + gc * s00
    gdet = -gdeti * deti * deti * c["dmask"]
    gs00 = gs00 + gdet * s11
    gs11 = gs11 + gdet * s00
    gs01 = gs01 + gdet * (-2 * s01)
    J00, J02, J11, J12 = c["J00"], c["J02"], c["J11"], c["J12"]
    SC = c["SC"]
    SC00, SC01, SC02, SC11, SC12, SC22 = SC[0][0], SC[0][1], SC[0][2], SC[1][1], SC[1][2], SC[2][2]
    gJ00 = gs00 * (2 * J00 * SC00 + 2 * J02 * SC02) + gs01 * (J11 * SC01 + J12 * SC02)
    gJ02 = gs00 * (2 * J00 * SC02 + 2 * J02 * SC22) + gs01 * (J11 * SC12 + J12 * SC22)
    gJ11 = gs11 * (2 * J11 * SC11 + 2 * J12 * SC12) + gs01 * (J00 * SC01 + J02 * SC12)
    gJ12 = gs11 * (2 * J11 * SC12 + 2 * J12 * SC22) + gs01 * (J00 * SC02 + J02 * SC22)
    gSC00 = gs00 * J00 * J00
    gSC11 = gs11 * J11 * J11
    gSC22 = gs00 * J02 * J02 + gs11 * J12 * J12 + gs01 * J02 * J12
    gSC02 = gs00 * 2 * J00 * J02 + gs01 * J00 * J12
    gSC12 = gs11 * 2 * J11 * J12 + gs01 * J02 * J11
    gSC01 = gs01 * J00 * J11
    fx, fy, mcx, mcy, zi = c["fx"], c["fy"], c["mcx"], c["mcy"], c["zi"]
    gmcx = gmux * fx * zi + gJ02 * (-fx * zi * zi)
    gmcy = gmuy * fy * zi + gJ12 * (-fy * zi * zi)
    gzi = (gmux * fx * mcx + gmuy * fy * mcy + gJ00 * fx + gJ11 * fy
           + gJ02 * (-fx * mcx * 2 * zi) + gJ12 * (-fy * mcy * 2 * zi))
    gmcz = -gzi * zi * zi * c["zmask"]
    Rv = c["Rv"]
    gmeans = np.stack([gmcx * Rv[0][i] + gmcy * Rv[1][i] + gmcz * Rv[2][i] for i in range(3)], -1)
    M, s2 = c["M"], c["s2"]
    zero = np.zeros_like(mcx)
    gM = [[zero.copy() for _ in range(3)] for _ in range(3)]
    gs2 = [zero.copy() for _ in range(3)]
    for gg, i in ((gSC00, 0), (gSC11, 1), (gSC22, 2)):
        for k in range(3):
            gM[i][k] = gM[i][k] + gg * 2 * M[i][k] * s2[k]
            gs2[k] = gs2[k] + gg * M[i][k] * M[i][k]
    for gg, i, l in ((gSC01, 0, 1), (gSC02, 0, 2), (gSC12, 1, 2)):
        for k in range(3):
            gM[i][k] = gM[i][k] + gg * M[l][k] * s2[k]
            gM[l][k] = gM[l][k] + gg * M[i][k] * s2[k]
            gs2[k] = gs2[k] + gg * M[i][k] * M[l][k]
    gscale = np.stack([gs2[0] * 2 * c["sx"], gs2[1] * 2 * c["sy"], gs2[2] * 2 * c["sz"]], -1)
    gR = [[Rv[0][i] * gM[0][k] + Rv[1][i] * gM[1][k] + Rv[2][i] * gM[2][k] for k in range(3)]
          for i in range(3)]
    w, x, y, z = c["w"], c["x"], c["y"], c["z"]
    (gR00, gR01, gR02), (gR10, gR11, gR12), (gR20, gR21, gR22) = gR
    gw = gR01 * (-2 * z) + gR02 * (2 * y) + gR10 * (2 * z) + gR12 * (-2 * x) + gR20 * (-2 * y) + gR21 * (2 * x)
    gx = (gR01 * (2 * y) + gR02 * (2 * z) + gR10 * (2 * y) + gR11 * (-4 * x) + gR12 * (-2 * w)
          + gR20 * (2 * z) + gR21 * (2 * w) + gR22 * (-4 * x))
    gy = (gR00 * (-4 * y) + gR01 * (2 * x) + gR02 * (2 * w) + gR10 * (2 * x) + gR12 * (2 * z)
          + gR20 * (-2 * w) + gR21 * (2 * z) + gR22 * (-4 * y))
    gz = (gR00 * (-4 * z) + gR01 * (-2 * w) + gR02 * (2 * x) + gR10 * (2 * w) + gR11 * (-4 * z)
          + gR12 * (2 * y) + gR20 * (2 * x) + gR21 * (2 * y))
    n = c["n"]
    dot = w * gw + x * gx + y * gy + z * gz
    gquat = np.stack([(gw - w * dot) / n, (gx - x * dot) / n, (gy - y * dot) / n, (gz - z * dot) / n], -1)
    return gmeans, gquat, gscale


def camera_center(cam):
    """Camera.center (spike/camera.py:46-48): -R_v^T t_v, float32 like the reference."""
    Rv = np.asarray(cam["R_v"], np.float32)
    tv = np.asarray(cam["t_v"], np.float32)
    return (-(Rv.T @ tv)).astype(np.float32)
