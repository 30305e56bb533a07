"""Oracle: the full binned render and train step composed from the restated pieces.

Per view (the reference's CPU path ``tools/m4_train_binned.py:189-230`` with the SH colour of
``spike/render.py:22-25``): geometry -> SH colour / activations -> assign_bins -> operands ->
binned WSR forward -> loss -> binned backward -> theta-build backward -> slot->gaussian
index_add -> geometry/SH/activation backward (``tools/operands_manual.py:83-110``).
Train step (``spike/mcmc.py:90-114``): mean of the per-view photometric losses plus the MCMC
regulariser, Adam (``spike/train.py:19,29``), SGLD noise, and relocation.
"""
import numpy as np

from . import binning, geometry, loss as loss_mod, optim, render, sh

F32 = np.float32
PARAM_NAMES = ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest")


def copy_params(p):
    out = {k: np.array(p[k], F32, copy=True) for k in PARAM_NAMES}
    out["w_b_raw"] = F32(p["w_b_raw"])
    return out


def colour_of(params, sh_degree, cam):
    """Per-gaussian RGB: eval_sh_color on means - camera centre (spike/render.py:22-25) or the
    DC-only colour (spike/forward.py:69-71).  Returns (colour f64, pre-clamp f64, dirs)."""
    dc = np.asarray(params["color_dc"], np.float64)
    if sh_degree > 0:
        coeffs = np.concatenate([dc[:, None, :], np.asarray(params["color_rest"], np.float64)], 1)
        dirs = np.asarray(params["means3d"], np.float32) - geometry.camera_center(cam)[None, :]
        col, pre = sh.eval_sh_color(sh_degree, coeffs, dirs)
        return col, pre, dirs
    pre = 0.5 + sh.C0 * dc
    return np.maximum(pre, 0.0), pre, None


def render_view(params, sh_degree, cam, K=128, R=1, k=4.0, blur=0.3, near=0.2, bins=None,
                c_b=(1.0, 1.0, 1.0), depth_bt=None, arm="A"):
    """Forward for one view; returns a dict with the image and everything the backward needs.
    ``depth_bt`` = (depth_beta, depth_tau) selects arm B (spike/arms.py:34-37): the opacity is
    scaled by rho = sigmoid(depth_beta (depth_tau - z)) of the camera-space z; ``arm="RV"`` blends
    with revealage compositing (spike/arms.py:70-83)."""
    conic, mu2d, depth, keep, gcache = geometry.fwd(params["means3d"], params["quats"],
                                                    params["log_scales"], cam, blur, near)
    mu2d32, conic32 = mu2d.astype(F32), conic.astype(F32)
    colour, pre, dirs = colour_of(params, sh_degree, cam)
    o = render.sigmoid(params["opacity_raw"]).astype(F32)
    rho = np.ones_like(o, dtype=np.float64)
    if depth_bt is not None:
        rho = render.sigmoid(float(depth_bt[0]) * (float(depth_bt[1]) - np.asarray(depth, np.float64)))
        o = (o * rho).astype(F32)
    tm = binning.tile_map(cam["H"], cam["W"])
    if bins is None:
        bins = binning.assign_bins(mu2d32, keep, tm, R, K)
    theta, col, oc, w_b = render.operands(mu2d32, conic32, keep, colour.astype(F32), o,
                                          params["w_b_raw"], bins, tm, k)
    if arm == "RV":
        img, den, rcache = render.render_fwd_rv(theta, col, oc, np.asarray(c_b, F32), tm)
    else:
        img, den, rcache = render.render_fwd(theta, col, oc, w_b, np.asarray(c_b, F32), tm)
    return dict(img=img, den=den, rcache=rcache, bins=bins, tm=tm, theta=theta, col=col, oc=oc,
                w_b=w_b, mu2d=mu2d32, conic=conic32, keep=keep, depth=depth, gcache=gcache,
                colour=colour, pre=pre, dirs=dirs, o=render.sigmoid(params["opacity_raw"]).astype(F32), rho=rho,
                depth_bt=depth_bt, c_b=np.asarray(c_b, F32), k=k, cam=cam, arm=arm)


def backward_view(fw, gimg, params, sh_degree):
    """Manual backward of ``render_view`` for dL/dimg; returns per-parameter grads (float64)."""
    tm, bins = fw["tm"], fw["bins"]
    G = params["means3d"].shape[0]
    if fw["arm"] == "RV":
        gtheta, gcol, goc, gw_b = render.render_bwd_rv(gimg, fw["theta"], fw["col"], fw["oc"], fw["c_b"], tm,
                                                       fw["rcache"])
    else:
        gtheta, gcol, goc, gw_b = render.render_bwd(gimg, fw["theta"], fw["col"], fw["oc"], fw["w_b"],
                                                    fw["c_b"], tm, fw["rcache"])
    conic_t, mu_t = fw["conic"][bins.idx], fw["mu2d"][bins.idx]
    gconic_t, gmu_t = render.theta_bwd(gtheta, conic_t, mu_t, tm.origins, bins.valid, fw["k"])
    g9 = render.scatter_slots(G, bins.idx, bins.valid, gconic_t, gmu_t, gcol, goc)
    gm, gq, gs = geometry.bwd(fw["gcache"], g9[:, 0], g9[:, 1], g9[:, 2], g9[:, 3], g9[:, 4])
    keepf = fw["keep"].astype(np.float64)
    o = fw["o"].astype(np.float64)
    rho = fw["rho"]
    keo = keepf * o * rho
    gcolor_o, go_col = g9[:, 5:8], g9[:, 8]
    gkeo = (gcolor_o * fw["colour"]).sum(-1) + go_col
    gcolour = gcolor_o * keo[:, None]
    gop = gkeo * keepf * rho * o * (1.0 - o)
    gdepth = None
    if fw["depth_bt"] is not None:
        beta, tau = float(fw["depth_bt"][0]), float(fw["depth_bt"][1])
        grho = gkeo * keepf * o * rho * (1.0 - rho)
        z = np.asarray(fw["depth"], np.float64)
        gdepth = (float((grho * (tau - z)).sum()), float((grho * beta).sum()))
        gm = gm + (-grho * beta)[:, None] * np.asarray(fw["cam"]["R_v"], np.float64)[2][None, :]
    grest = np.zeros((G, 15, 3))
    if sh_degree > 0:
        coeffs = np.concatenate([np.asarray(params["color_dc"], np.float64)[:, None, :],
                                 np.asarray(params["color_rest"], np.float64)], 1)
        gco, gdirs = sh.eval_sh_color_bwd(sh_degree, coeffs, fw["dirs"], gcolour)
        gm = gm + gdirs
        gdc = gco[:, 0]
        grest[:, :gco.shape[1] - 1] = gco[:, 1:]
    else:
        gdc = gcolour * sh.C0 * (fw["pre"] >= 0.0)
    out = dict(means3d=gm, log_scales=gs * fw["gcache"]["scale"], quats=gq, opacity_raw=gop,
               color_dc=gdc, color_rest=grest,
               w_b_raw=float(gw_b) * float(render.sigmoid(params["w_b_raw"])))
    if gdepth is not None:
        out["depth_beta"], out["depth_tau"] = gdepth
    return out


def loss_and_grads(params, cams, targets, sh_degree, K=128, R=1, k=4.0, lam=0.2,
                   lambda_o=0.0, lambda_s=0.0, depth_bt=None, arm="A"):
    """Mean over views of loss_fn (spike/train.py:24-27) + reg_loss (spike/mcmc.py:102); returns
    (total loss, per-view losses, grads dict)."""
    V = len(cams)
    grads = None
    losses = []
    for cam, tgt in zip(cams, targets):
        fw = render_view(params, sh_degree, cam, K, R, k, depth_bt=depth_bt, arm=arm)
        lv, _, _, gimg = loss_mod.loss_and_grad(fw["img"], tgt, lam)
        losses.append(lv)
        gv = backward_view(fw, (gimg / V).astype(F32), params, sh_degree)
        grads = gv if grads is None else {n: grads[n] + gv[n] for n in grads}
    total = float(np.mean(losses))
    if lambda_o or lambda_s:
        gop, gls = optim.reg_loss_grads(params["opacity_raw"], params["log_scales"], lambda_o, lambda_s)
        grads["opacity_raw"] = grads["opacity_raw"] + gop
        grads["log_scales"] = grads["log_scales"] + gls
        o = render.sigmoid(params["opacity_raw"])
        s = np.exp(np.asarray(params["log_scales"], np.float64))
        total += lambda_o * o.mean() + lambda_s * s.mean()
    return total, losses, grads


def lr_of(lr):
    """Per-parameter learning rates of GaussianModel.param_groups (spike/model.py:82-95)."""
    return dict(means3d=lr["means"], log_scales=lr["scales"], quats=lr["quats"],
                opacity_raw=lr["opacity"], color_dc=lr["color"],
                color_rest=lr.get("color_rest", lr["color"] / 20.0), w_b_raw=lr["wb"])


def adam_step(params, grads, state, step, lr, sh_degree):
    """torch.optim.Adam over the parameters that receive a gradient (colour rest only when the
    SH degree is above 0, as torch skips parameters whose .grad is None)."""
    lrs = lr_of(lr)
    for name in PARAM_NAMES + ("w_b_raw",):
        if name == "color_rest" and sh_degree == 0:
            continue
        p = np.atleast_1d(np.asarray(params[name], F32)).copy()
        g = np.atleast_1d(np.asarray(grads[name], F32))
        m, v = state.setdefault(name, (np.zeros_like(p), np.zeros_like(p)))
        optim.adam_update(p, g, m, v, step, lrs[name])
        params[name] = p if name != "w_b_raw" else F32(p[0])
