"""Oracle: per-tile operands, the binned poly-splat + WSR forward and its manual backward.

Restates, in float32 numpy:
- ``theta_u_gathered`` (tools/m4_train_binned.py:130-143) in the reference's exact op order;
- the operand gather/mask of ``_operands`` (tools/m4_train_binned.py:198-212);
- the binned forward ``render_binned_cpu`` (tools/m4_train_binned.py:226-230), i.e.
  ``WSRPolySplatHot.forward`` (spike/backward.py:28-41) per tile;
- the binned backward ``_DevRenderBinned.backward`` (tools/m4_train_binned.py:169-186), i.e.
  ``WSRPolySplatHot.backward`` (spike/backward.py:43-58) per tile;
- the theta-build backward ``_theta_bwd`` (tools/operands_manual.py:65-80) and the slot ->
  gaussian ``index_add`` (tools/operands_manual.py:94-98);
- the dense reference ``wsr_polysplat_ref`` (spike/backward.py:11-20) and its manual backward,
  for the dense entry point.
"""
import numpy as np

F32 = np.float32


def softplus(x):
    """torch.nn.functional.softplus (beta 1, threshold 20)."""
    x = np.asarray(x, np.float64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))


def theta_u_gathered(conic_t, mu_t, origins, k):
    """tools/m4_train_binned.py:130-143, fp32 op order: conic_t[T,K,3], mu_t[T,K,2],
    origins[T,2] -> theta_u[T,6,K] (tile origin folded into the mean)."""
    conic_t = np.asarray(conic_t, F32)
    mu = np.asarray(mu_t, F32) - np.asarray(origins, F32)[:, None, :]
    a, b, c = conic_t[..., 0], conic_t[..., 1], conic_t[..., 2]
    mux, muy = mu[..., 0], mu[..., 1]
    ik = F32(1.0 / k)
    two = F32(2.0)
    Q = ((a * mux) * mux + ((two * b) * mux) * muy) + (c * muy) * muy
    th = np.stack([
        (-a) * ik, (-c) * ik, (F32(-2.0) * b) * ik,
        (two * (a * mux + b * muy)) * ik,
        (two * (b * mux + c * muy)) * ik,
        F32(1.0) - Q * ik], -1)
    return np.ascontiguousarray(np.transpose(th, (0, 2, 1)))


def operands(mu2d, conic, keep, color, o, w_b_raw, bins, tm, k=4.0):
    """_operands' gather + mask (tools/m4_train_binned.py:198-212) given per-gaussian
    activations: -> theta_u[T,6,K], color_o_t[T,K,3], o_col_t[T,K,1], w_b."""
    keo = (np.asarray(keep, F32) * np.asarray(o, F32))[:, None]
    color_o = keo * np.asarray(color, F32)
    o_col = keo
    idx, valid = bins.idx, bins.valid
    vf = valid[..., None].astype(F32)
    conic_t = np.asarray(conic, F32)[idx]
    mu_t = np.asarray(mu2d, F32)[idx]
    theta = theta_u_gathered(conic_t, mu_t, tm.origins, k) * valid[:, None, :].astype(F32)
    return theta, color_o[idx] * vf, o_col[idx] * vf, F32(softplus(w_b_raw))


def render_fwd(theta, col, oc, w_b, c_b, tm):
    """Binned forward (tools/m4_train_binned.py:226-230): -> img[H,W,3], den[H,W] and the
    per-tile intermediates (relu_Q, w, C) the backward recomputes."""
    T = theta.shape[0]
    u = np.matmul(tm.Phi[None], theta)                          # [T,256,K]
    relu = np.maximum(u, F32(0.0))
    w = relu * relu
    c_b = np.asarray(c_b, F32)
    num = np.matmul(w, col) + F32(w_b) * c_b                     # [T,256,3]
    den = np.matmul(w, oc) + F32(w_b)                            # [T,256,1]
    C = num / den
    img = np.zeros((tm.H * tm.W, 3), F32)
    img[tm.gidx] = C.reshape(-1, 3)
    den_img = np.zeros(tm.H * tm.W, F32)
    den_img[tm.gidx] = den.reshape(-1)
    return img.reshape(tm.H, tm.W, 3), den_img.reshape(tm.H, tm.W), (relu, w, C, den)


def render_bwd(gimg, theta, col, oc, w_b, c_b, tm, cache=None):
    """_DevRenderBinned.backward (tools/m4_train_binned.py:169-186) in fp32:
    -> gtheta[T,6,K], gcol[T,K,3], goc[T,K,1], gw_b (scalar)."""
    T = theta.shape[0]
    if cache is None:
        _, _, cache = render_fwd(theta, col, oc, w_b, c_b, tm)
    relu, w, C, den = cache
    gC = np.asarray(gimg, F32).reshape(-1, 3)[tm.gidx].reshape(T, 256, 3)
    gnum = gC / den
    gden = -np.sum(gC * C, -1, keepdims=True) / den
    wT = np.transpose(w, (0, 2, 1))
    gcol = np.matmul(wT, gnum)
    goc = np.matmul(wT, gden)
    gw = np.matmul(gnum, np.transpose(col, (0, 2, 1))) + np.matmul(gden, np.transpose(oc, (0, 2, 1)))
    gtheta = np.matmul(tm.Phi.T[None], gw * (relu * F32(2.0)))
    c_b = np.asarray(c_b, F32)
    gw_b = F32(np.sum(gnum * c_b[None, None, :], dtype=np.float64) + np.sum(gden, dtype=np.float64))
    return gtheta, gcol, goc, gw_b


RV_EPS = F32(1e-6)
RV_AMAX = F32(1.0 - 1e-4)


def render_fwd_rv(theta, col, oc, c_b, tm):
    """Binned arm RV (blend_RV, spike/arms.py:70-83, on the tile operands) in fp32:
    W = w oc, den = sum W + eps, Cavg = sum w col / den, R = exp(sum log1p(-clamp(W, 0, 1-1e-4))),
    C = Cavg (1 - R) + c_b R.  -> img[H,W,3], den[H,W], cache."""
    u = np.matmul(tm.Phi[None], theta)                          # [T,256,K]
    relu = np.maximum(u, F32(0.0))
    w = relu * relu
    Wm = w * np.transpose(oc, (0, 2, 1))                         # [T,256,K]
    den = np.matmul(w, oc) + RV_EPS                              # [T,256,1]
    Cavg = np.matmul(w, col) / den
    a = np.clip(Wm, F32(0.0), RV_AMAX)
    R = np.exp(np.sum(np.log1p(-a), -1, keepdims=True))         # [T,256,1]
    c_b = np.asarray(c_b, F32)
    C = Cavg * (F32(1.0) - R) + c_b[None, None, :] * R
    img = np.zeros((tm.H * tm.W, 3), F32)
    img[tm.gidx] = C.reshape(-1, 3)
    den_img = np.zeros(tm.H * tm.W, F32)
    den_img[tm.gidx] = den.reshape(-1)
    return img.reshape(tm.H, tm.W, 3), den_img.reshape(tm.H, tm.W), (relu, w, Wm, Cavg, den, R)


def render_bwd_rv(gimg, theta, col, oc, c_b, tm, cache=None):
    """Manual backward of ``render_fwd_rv`` (the autograd of blend_RV restated per tile):
    -> gtheta[T,6,K], gcol[T,K,3], goc[T,K,1], gw_b = 0 (w_b does not enter the blend)."""
    T = theta.shape[0]
    if cache is None:
        _, _, cache = render_fwd_rv(theta, col, oc, c_b, tm)
    relu, w, Wm, Cavg, den, R = cache
    c_b = np.asarray(c_b, F32)
    gC = np.asarray(gimg, F32).reshape(-1, 3)[tm.gidx].reshape(T, 256, 3)
    f = (F32(1.0) - R) / den
    gnum = gC * f
    gden = -np.sum(gC * Cavg, -1, keepdims=True) * f
    gL = R * np.sum(gC * (c_b[None, None, :] - Cavg), -1, keepdims=True)
    inside = (Wm >= 0) & (Wm <= RV_AMAX)                          # clamp passes no gradient outside
    gW = gden - np.where(inside, gL / (F32(1.0) - np.clip(Wm, F32(0.0), RV_AMAX)), F32(0.0))  # [T,256,K]
    wT = np.transpose(w, (0, 2, 1))
    gcol = np.matmul(wT, gnum)
    goc = np.sum(gW * w, 1)[..., None]
    gw = np.matmul(gnum, np.transpose(col, (0, 2, 1))) + gW * np.transpose(oc, (0, 2, 1))
    gtheta = np.matmul(tm.Phi.T[None], gw * (relu * F32(2.0)))
    return gtheta, gcol, goc, F32(0.0)


def theta_bwd(gtheta, conic_t, mu_t, origins, valid, k=4.0):
    """_theta_bwd (tools/operands_manual.py:65-80): gtheta[T,6,K] -> gconic_t[T,K,3],
    gmu_t[T,K,2], masked by valid.  Computed in float64."""
    T, K = conic_t.shape[0], conic_t.shape[1]
    gpoly = np.transpose(np.asarray(gtheta, np.float64) * valid[:, None, :], (0, 2, 1))
    gtQ = gpoly * (-1.0 / k)
    g0, g1, g2, g3, g4, g5 = (gtQ[..., j] for j in range(6))
    conic_t = np.asarray(conic_t, np.float64)
    a, b, c = conic_t[..., 0], conic_t[..., 1], conic_t[..., 2]
    mu = np.asarray(mu_t, np.float64) - np.asarray(origins, np.float64)[:, None, :]
    mux, muy = mu[..., 0], mu[..., 1]
    ga = g0 + g3 * (-2 * mux) + g5 * mux * mux
    gb = 2 * g2 + g3 * (-2 * muy) + g4 * (-2 * mux) + g5 * (2 * mux * muy)
    gc = g1 + g4 * (-2 * muy) + g5 * muy * muy
    gmux = g3 * (-2 * a) + g4 * (-2 * b) + g5 * (2 * a * mux + 2 * b * muy)
    gmuy = g3 * (-2 * b) + g4 * (-2 * c) + g5 * (2 * b * mux + 2 * c * muy)
    return np.stack([ga, gb, gc], -1), np.stack([gmux, gmuy], -1)


def scatter_slots(G, idx, valid, gconic_t, gmu_t, gcol, goc):
    """index_add of per-slot grads into per-gaussian grads (tools/operands_manual.py:94-98),
    every channel masked by valid: -> [G,9] = (ga, gb, gc, gmux, gmuy, gcol_o[3], go_col)."""
    vf = valid[..., None].astype(np.float64)
    g9 = np.concatenate([gconic_t * vf, gmu_t * vf, np.asarray(gcol, np.float64) * vf,
                         np.asarray(goc, np.float64) * vf], -1).reshape(-1, 9)
    out = np.zeros((G, 9), np.float64)
    np.add.at(out, idx.reshape(-1), g9)
    return out


def wsr_dense_fwd(theta_u, o, color, w_b, Phi, c_b, keep=None):
    """wsr_polysplat_ref (spike/backward.py:11-20), float64: theta_u[G,6], Phi[P,6] -> C[P,3]."""
    u = np.asarray(Phi, np.float64) @ np.asarray(theta_u, np.float64).T
    relu = np.maximum(u, 0.0)
    wg = relu * relu
    if keep is not None:
        wg = wg * np.asarray(keep, np.float64)[None, :]
    w = np.asarray(o, np.float64)[None, :] * wg
    num = w @ np.asarray(color, np.float64) + float(w_b) * np.asarray(c_b, np.float64)[None, :]
    den = w.sum(1, keepdims=True) + float(w_b)
    return num / den


def wsr_dense_bwd(gC, theta_u, o, color, w_b, Phi, c_b, keep=None):
    """WSRPolySplatHot.backward (spike/backward.py:43-58), float64 ->
    (gtheta[G,6], go[G], gcolor[G,3], gw_b)."""
    Phi = np.asarray(Phi, np.float64)
    u = Phi @ np.asarray(theta_u, np.float64).T
    relu = np.maximum(u, 0.0)
    wg = relu * relu
    kf = np.ones(u.shape[1]) if keep is None else np.asarray(keep, np.float64)
    wg = wg * kf[None, :]
    o = np.asarray(o, np.float64)
    color = np.asarray(color, np.float64)
    w = o[None, :] * wg
    num = w @ color + float(w_b) * np.asarray(c_b, np.float64)[None, :]
    den = w.sum(1, keepdims=True) + float(w_b)
    C = num / den
    gC = np.asarray(gC, np.float64)
    inv = 1.0 / den
    gnum = gC * inv
    gden = -(gC * C).sum(1, keepdims=True) * inv
    gw = gnum @ color.T + gden
    gcolor = w.T @ gnum
    gw_b = (gnum * np.asarray(c_b, np.float64)[None, :]).sum() + gden.sum()
    go = (gw * wg).sum(0)
    gu = gw * o[None, :] * kf[None, :] * (2.0 * relu)
    gtheta = gu.T @ Phi
    return gtheta, go, gcolor, gw_b
