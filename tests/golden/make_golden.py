"""Generate the golden fixtures by running the reference implementation itself.

Usage (build container only; the reference checkout does not exist on GPU boxes):

    python tests/golden/make_golden.py --reference <path to the kinginu/tt-splat checkout>

The reference's CPU torch path is imported unmodified.  Two third-party modules it imports at
module top are replaced by empty stubs in ``sys.modules`` before import: ``ttnn`` (Tenstorrent
runtime; unused by the functions called here) and ``pytorch_msssim`` (not installed; only the
SSIM of ``spike/metrics.py`` calls it, and no fixture here goes through that function).
Every fixture stores its inputs next to the reference's outputs, so tests never need the
reference.  Inputs come from ``tt-splat_b200/synthetic.py`` (seeded numpy).

``render_binned_cpu`` (tools/m4_train_binned.py:222-230) cannot be called as is (it unpacks the
five values of ``_operands`` into four names); its three lines of math are applied here to the
output of the reference's own ``_operands``.
"""
import argparse
import hashlib
import importlib.util
import os
import sys
import types

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)

from make_golden_cases import BIG_CASE, RADIUS_CASES, STRESS_CASES  # noqa: E402


def load_synthetic():
    spec = importlib.util.spec_from_file_location("_synthetic", os.path.join(REPO, "tt-splat_b200", "synthetic.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def import_reference(ref):
    sys.modules.setdefault("ttnn", types.ModuleType("ttnn"))
    pm = types.ModuleType("pytorch_msssim")

    def _absent(*a, **k):
        raise RuntimeError("pytorch_msssim is not installed")
    pm.ssim = _absent
    sys.modules.setdefault("pytorch_msssim", pm)
    sys.path.insert(0, ref)
    sys.path.insert(0, os.path.join(ref, "tools"))
    from spike import camera, geometry, mcmc, sh  # noqa: F401
    import geom_bwd
    import loss_manual
    import m4_train_binned as mb
    return types.SimpleNamespace(camera=camera, geometry=geometry, mcmc=mcmc, sh=sh, mb=mb,
                                 geom_bwd=geom_bwd, loss_manual=loss_manual)


class _StableArgsort:
    """Context manager forcing torch.argsort(stable=True): the canonical binning order."""

    def __enter__(self):
        self.orig = torch.argsort
        orig = self.orig
        torch.argsort = lambda x, *a, **k: orig(x, *a, **{**k, "stable": True})

    def __exit__(self, *exc):
        torch.argsort = self.orig


def t(x, grad=False):
    out = torch.tensor(np.asarray(x), dtype=torch.float32)
    return out.requires_grad_(grad)


def ref_cam(R, cam):
    return R.camera.Camera(t(cam["R_v"]), t(cam["t_v"]), cam["fx"], cam["fy"], cam["cx"], cam["cy"],
                           cam["H"], cam["W"])


def cam_arrays(cam, prefix="cam_"):
    return {prefix + "R_v": cam["R_v"], prefix + "t_v": cam["t_v"],
            prefix + "intr": np.array([cam["fx"], cam["fy"], cam["cx"], cam["cy"]], np.float64),
            prefix + "hw": np.array([cam["H"], cam["W"]], np.int64)}


def project(R, p, cam):
    Rm = R.geometry.quat_to_rotmat(t(p["quats"]))
    cov = R.geometry.cov3d(torch.exp(t(p["log_scales"])), Rm)
    return R.geometry.project_ewa(t(p["means3d"]), cov, t(cam["R_v"]), t(cam["t_v"]),
                                  cam["fx"], cam["fy"], cam["cx"], cam["cy"], 0.3, 0.2)


def bins_of(R, mu2d, keep, H, W, Rr, K, stable):
    tmap = R.mb.TileMap(H, W)
    if stable:
        with _StableArgsort():
            idx, valid = R.mb.assign_bins(mu2d, keep, tmap, Rr, K)
    else:
        idx, valid = R.mb.assign_bins(mu2d, keep, tmap, Rr, K)
    return idx.numpy(), valid.numpy()


def digest(idx, valid, cand):
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(np.where(valid, idx, -1).astype(np.int32)).tobytes())
    h.update(np.ascontiguousarray(valid.sum(1).astype(np.int32)).tobytes())
    h.update(np.ascontiguousarray(cand.astype(np.int32)).tobytes())
    return h.hexdigest()


def cand_of(R, mu2d, keep, H, W, Rr):
    """Candidates per tile from the reference: assign_bins with K above every candidate count
    keeps everything, so valid.sum(1) is the candidate count."""
    K = 64
    while True:
        idx, valid = bins_of(R, mu2d, keep, H, W, Rr, K, True)
        c = valid.sum(1)
        if c.max() < K:
            return c.astype(np.int64)
        K *= 4


def gen_bins_scene(R, syn, out):
    sc = syn.config0()
    p, cam = sc["params"], sc["cams"][0]
    mu2d, conic, depth, keep = project(R, p, cam)
    idx_s, valid_s = bins_of(R, mu2d, keep, cam["H"], cam["W"], 1, 128, True)
    idx_d, valid_d = bins_of(R, mu2d, keep, cam["H"], cam["W"], 1, 128, False)
    np.savez_compressed(os.path.join(out, "bins_config0.npz"), mu2d=mu2d.numpy(), keep=keep.numpy(),
                        conic=conic.numpy(), depth=depth.numpy(), idx_stable=idx_s.astype(np.int32),
                        valid_stable=valid_s, idx_default=idx_d.astype(np.int32), valid_default=valid_d,
                        cand=cand_of(R, mu2d, keep, cam["H"], cam["W"], 1).astype(np.int32),
                        K=128, R=1, **cam_arrays(cam), **{k: v for k, v in p.items() if k != "color_rest"})

    sc = syn.config1()
    p, cam = sc["params"], sc["cams"][0]
    mu2d, conic, depth, keep = project(R, p, cam)
    idx_s, valid_s = bins_of(R, mu2d, keep, cam["H"], cam["W"], 1, 128, True)
    cand = cand_of(R, mu2d, keep, cam["H"], cam["W"], 1)
    np.savez_compressed(os.path.join(out, "bins_config1.npz"), mu2d=mu2d.numpy(), keep=keep.numpy(),
                        digest=digest(idx_s, valid_s, cand), cand=cand.astype(np.int32),
                        full_tiles=int((valid_s.sum(1) == 128).sum()), K=128, R=1, **cam_arrays(cam))




def gen_bins_stress(R, syn, out, cases=STRESS_CASES, fname="bins_stress.npz"):
    arrays = {}
    for name, seed, G, H, W, Rr, K, kw in cases:
        mu, keep = syn.stress_mu2d(seed, G, H, W, **kw)
        idx_s, valid_s = bins_of(R, torch.from_numpy(mu), torch.from_numpy(keep), H, W, Rr, K, True)
        idx_d, valid_d = bins_of(R, torch.from_numpy(mu), torch.from_numpy(keep), H, W, Rr, K, False)
        cand = cand_of(R, torch.from_numpy(mu), torch.from_numpy(keep), H, W, Rr)
        arrays.update({f"{name}__idx_stable": idx_s.astype(np.int32), f"{name}__valid_stable": valid_s,
                       f"{name}__idx_default": idx_d.astype(np.int32), f"{name}__valid_default": valid_d,
                       f"{name}__cand": cand.astype(np.int32)})
    np.savez_compressed(os.path.join(out, fname), **arrays)


def gen_bins_big(R, syn, out):
    c = BIG_CASE
    mu, keep = syn.stress_mu2d(c["seed"], c["G"], c["H"], c["W"], **c["kw"])
    mt, kt = torch.from_numpy(mu), torch.from_numpy(keep)
    idx_s, valid_s = bins_of(R, mt, kt, c["H"], c["W"], c["R"], c["K"], True)
    cand = cand_of(R, mt, kt, c["H"], c["W"], c["R"])
    np.savez_compressed(os.path.join(out, "bins_big.npz"), digest=digest(idx_s, valid_s, cand),
                        cand=cand.astype(np.int32), overflow=int(np.maximum(cand - c["K"], 0).sum()),
                        full_tiles=int((valid_s.sum(1) == c["K"]).sum()),
                        mu_sha=hashlib.sha256(mu.tobytes()).hexdigest())


class _Model:
    pass


def make_model(p, sh):
    m = _Model()
    for k in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc"):
        setattr(m, k, t(p[k], True))
    m.color_rest = t(p["color_rest"], True)
    m.w_b_raw = torch.tensor(float(p["w_b_raw"]), requires_grad=True)
    m.c_b = torch.ones(3)
    return m


def operands_sh(R, model, cam, tmap, Rr, K, sh_degree, cached_bins):
    """tools/m4_train_binned.py:189-212 with the SH colour of spike/render.py:22-25."""
    geometry, sh = R.geometry, R.sh
    Rm = geometry.quat_to_rotmat(model.quats)
    cov = geometry.cov3d(torch.exp(model.log_scales), Rm)
    mu2d, conic, depth, keep = geometry.project_ewa(model.means3d, cov, cam.R_v, cam.t_v, cam.fx, cam.fy,
                                                    cam.cx, cam.cy, 0.3, 0.2)
    coeffs = torch.cat([model.color_dc[:, None, :], model.color_rest], dim=1)
    color = sh.eval_sh_color(sh_degree, coeffs, model.means3d - cam.center[None, :])
    o = torch.sigmoid(model.opacity_raw)
    w_b = F.softplus(model.w_b_raw)
    keo = (keep.float() * o)[:, None]
    color_o, o_col = keo * color, keo
    idx, valid = cached_bins
    vf = valid[..., None].float()
    conic_t, mu_t = conic[idx], mu2d[idx]
    theta_u = R.mb.theta_u_gathered(conic_t, mu_t, tmap.origins, R.mb.K_POLY) * valid[:, None, :].float()
    return theta_u, color_o[idx] * vf, o_col[idx] * vf, w_b, (idx, valid)


def binned_render_and_grads(R, p, cam, target, K, sh_degree):
    model = make_model(p, sh_degree)
    rc = ref_cam(R, cam)
    tmap = R.mb.TileMap(cam["H"], cam["W"])
    with torch.no_grad():
        mu2d, _, _, keep = project(R, p, cam)
    with _StableArgsort():
        bins = R.mb.assign_bins(mu2d, keep, tmap, 1, K)
    if sh_degree == 0:
        thU, col, oc, w_b, _ = R.mb._operands(model, rc, tmap, 1, K, cached_bins=bins)
    else:
        thU, col, oc, w_b, _ = operands_sh(R, model, rc, tmap, 1, K, sh_degree, bins)
    for x in (thU, col, oc, w_b):
        x.retain_grad()
    # tools/m4_train_binned.py:226-230
    w = torch.relu(torch.einsum("pf,tfg->tpg", tmap.Phi, thU)) ** 2
    den = w @ oc + w_b
    C = (w @ col + w_b * model.c_b) / den
    img = torch.zeros(cam["H"] * cam["W"], 3)
    img[tmap.gidx] = C.reshape(-1, 3)
    img = img.reshape(cam["H"], cam["W"], 3)
    loss = (img - t(target)).abs().mean()
    loss.backward()
    g = {f"grad_{k}": getattr(model, k).grad.numpy() for k in
         ("means3d", "log_scales", "quats", "opacity_raw", "color_dc")}
    if sh_degree > 0:
        g["grad_color_rest"] = model.color_rest.grad.numpy()
    g["grad_w_b_raw"] = np.float32(model.w_b_raw.grad)
    den_img = torch.zeros(cam["H"] * cam["W"])
    den_img[tmap.gidx] = den.detach().reshape(-1)
    return dict(img=img.detach().numpy(), den=den_img.numpy().reshape(cam["H"], cam["W"]),
                loss=np.float64(loss.item()), theta_u=thU.detach().numpy(), col=col.detach().numpy(),
                oc=oc.detach().numpy(), w_b=np.float32(w_b.item()), gtheta=thU.grad.numpy(),
                gcol=col.grad.numpy(), goc=oc.grad.numpy(), gw_b=np.float32(w_b.grad),
                idx=bins[0].numpy().astype(np.int32), valid=bins[1].numpy(), **g)


def gen_render(R, syn, out):
    sc = syn.config0()
    p, cam, tgt = sc["params"], sc["cams"][0], sc["targets"][0]
    res = binned_render_and_grads(R, p, cam, tgt, 128, 0)
    np.savez_compressed(os.path.join(out, "render_config0.npz"), target=tgt, sh_degree=0, K=128,
                        **cam_arrays(cam), **{k: v for k, v in p.items() if k != "color_rest"}, **res)
    # SH degree 3, clustered (overflowing tiles), small image
    sc = syn.config1(seed=21, G=3000, res=128)
    p, cam, tgt = sc["params"], sc["cams"][0], sc["targets"][0]
    res = binned_render_and_grads(R, p, cam, tgt, 64, 3)
    np.savez_compressed(os.path.join(out, "render_sh3.npz"), target=tgt, sh_degree=3, K=64,
                        **cam_arrays(cam), **p, **res)


def gen_arm_b(R, syn, out):
    """Arm B (spike/arms.py:34-37: o * sigmoid(depth_beta * (depth_tau - depth))) through the
    reference's dense render (spike/render.py:14-49) on a scene whose tiles do not overflow K = 256
    and whose gaussians stay inside their 3x3 stencil, so the binned path must agree with it."""
    from spike import render as ref_render
    sc = syn.config0(seed=31, G=150, res=64)
    p, cam, tgt = sc["params"], sc["cams"][0], sc["targets"][0]
    out_arrays = {}
    for deg, tag in ((0, "deg0"), (3, "deg3")):
        model = make_model(p, deg)
        model.depth_beta = torch.tensor(1.3, requires_grad=True)
        model.depth_tau = torch.tensor(3.9, requires_grad=True)
        img = ref_render.render(model, ref_cam(R, cam), "B", sh_degree=deg)
        wts = torch.from_numpy(np.random.default_rng(32).standard_normal(img.shape).astype(np.float32))
        (img * wts).sum().backward()
        out_arrays[f"{tag}__img"] = img.detach().numpy()
        for k in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest"):
            gk = getattr(model, k).grad
            out_arrays[f"{tag}__grad_{k}"] = (gk if gk is not None else torch.zeros_like(getattr(model, k))).numpy()
        out_arrays[f"{tag}__grad_w_b_raw"] = np.float32(model.w_b_raw.grad)
        out_arrays[f"{tag}__grad_depth_beta"] = np.float32(model.depth_beta.grad)
        out_arrays[f"{tag}__grad_depth_tau"] = np.float32(model.depth_tau.grad)
        out_arrays["wts"] = wts.numpy()
    with torch.no_grad():
        mu2d, _, _, keep = project(R, p, cam)
    cand = cand_of(R, mu2d, keep, cam["H"], cam["W"], 1)
    assert int(cand.max()) <= 256, int(cand.max())
    np.savez_compressed(os.path.join(out, "render_arm_b.npz"), depth_beta=np.float32(1.3), depth_tau=np.float32(3.9),
                        K=256, **cam_arrays(cam), **p, **out_arrays)


def gen_arm_rv(R, syn, out):
    """Arm RV (revealage compositing, spike/arms.py:70-83) through the reference's dense render on
    the arm-B scene (tiles within K = 256, gaussians inside their stencil); a few gaussians get an
    opacity near 1 so that some pixel weights pass the 1 - 1e-4 clamp bound."""
    from spike import render as ref_render
    sc = syn.config0(seed=31, G=150, res=64)
    p, cam = dict(sc["params"]), sc["cams"][0]
    op = p["opacity_raw"].copy()
    op[:6] = 14.0
    p["opacity_raw"] = op
    # move those six onto pixel centres (x = col + 0.5, y = row + 0.5) at their camera depth, so
    # that their weight at that pixel is ~o > 1 - 1e-4
    Rv, tv = np.asarray(cam["R_v"], np.float64), np.asarray(cam["t_v"], np.float64)
    m = p["means3d"].astype(np.float64).copy()
    for i in range(6):
        mc = Rv @ m[i] + tv
        with torch.no_grad():
            mu = project(R, dict(p, means3d=m.astype(np.float32)), cam)[0][i].numpy().astype(np.float64)
        tx, ty = np.floor(mu[0]) + 0.5, np.floor(mu[1]) + 0.5
        mc[0] = (tx - cam["cx"]) * mc[2] / cam["fx"]
        mc[1] = (ty - cam["cy"]) * mc[2] / cam["fy"]
        m[i] = Rv.T @ (mc - tv)
    p["means3d"] = m.astype(np.float32)
    out_arrays = {}
    for deg, tag in ((0, "deg0"), (3, "deg3")):
        model = make_model(p, deg)
        img = ref_render.render(model, ref_cam(R, cam), "RV", sh_degree=deg)
        wts = torch.from_numpy(np.random.default_rng(33).standard_normal(img.shape).astype(np.float32))
        (img * wts).sum().backward()
        out_arrays[f"{tag}__img"] = img.detach().numpy()
        for k in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest"):
            gk = getattr(model, k).grad
            out_arrays[f"{tag}__grad_{k}"] = (gk if gk is not None else torch.zeros_like(getattr(model, k))).numpy()
        out_arrays["wts"] = wts.numpy()
    with torch.no_grad():
        mu2d, _, _, keep = project(R, p, cam)
    cand = cand_of(R, mu2d, keep, cam["H"], cam["W"], 1)
    assert int(cand.max()) <= 256, int(cand.max())
    np.savez_compressed(os.path.join(out, "render_arm_rv.npz"), K=256, **cam_arrays(cam), **p, **out_arrays)


def gen_sh12(R, syn, out):
    """Arm A at SH degrees 1 and 2 through the reference's dense render on the arm-B scene (tiles
    within K = 256, gaussians inside their stencil), with non-zero rest coefficients."""
    from spike import render as ref_render
    sc = syn.config0(seed=31, G=150, res=64)
    p, cam = dict(sc["params"]), sc["cams"][0]
    p["color_rest"] = (0.3 * np.random.default_rng(34).standard_normal((p["means3d"].shape[0], 15, 3))).astype(np.float32)
    out_arrays = {}
    for deg in (1, 2):
        model = make_model(p, deg)
        img = ref_render.render(model, ref_cam(R, cam), "A", sh_degree=deg)
        wts = torch.from_numpy(np.random.default_rng(35).standard_normal(img.shape).astype(np.float32))
        (img * wts).sum().backward()
        out_arrays[f"deg{deg}__img"] = img.detach().numpy()
        for k in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest"):
            gk = getattr(model, k).grad
            out_arrays[f"deg{deg}__grad_{k}"] = (gk if gk is not None else torch.zeros_like(getattr(model, k))).numpy()
        out_arrays[f"deg{deg}__grad_w_b_raw"] = np.float32(model.w_b_raw.grad)
        out_arrays["wts"] = wts.numpy()
    np.savez_compressed(os.path.join(out, "render_sh12.npz"), K=256, **cam_arrays(cam), **p, **out_arrays)


def gen_geom(R, syn, out):
    sc = syn.config0(seed=5, G=500)
    p, cam = sc["params"], sc["cams"][0]
    gb = R.geom_bwd
    means, quat, logs = t(p["means3d"], True), t(p["quats"], True), t(p["log_scales"], True)
    Rv = [[float(cam["R_v"][i, j]) for j in range(3)] for i in range(3)]
    tv = [float(x) for x in cam["t_v"]]
    conic, mu, _ = gb.fwd(means, quat, torch.exp(logs), Rv, tv, cam["fx"], cam["fy"], cam["cx"], cam["cy"])
    g = torch.Generator().manual_seed(0)
    gconic = torch.randn(conic.shape, generator=g)
    gmu = torch.randn(mu.shape, generator=g)
    ((conic * gconic).sum() + (mu * gmu).sum()).backward()
    np.savez_compressed(os.path.join(out, "geom_bwd.npz"), means3d=p["means3d"], quats=p["quats"],
                        log_scales=p["log_scales"], conic=conic.detach().numpy(), mu2d=mu.detach().numpy(),
                        gconic=gconic.numpy(), gmu=gmu.numpy(), gmeans=means.grad.numpy(),
                        gquats=quat.grad.numpy(), glog_scales=logs.grad.numpy(), **cam_arrays(cam))


def gen_near_plane(R, syn, out):
    """Thin gaussians just past the near plane whose means project far off-screen: the reference's
    fp32 project_ewa (spike/geometry.py:28-57) evaluates det = s00 s11 - s01^2 of a nearly rank-one
    Sigma2d as rounding noise and clamps it to 1e-12 for some of them (conics of ~1e20), although
    det(J Sigma J^T + blur I) >= blur^2 exactly.  Seeded needles on the config-2 view-1 camera;
    kept: every needle whose reference conic exceeds 1e6 (up to 32) and 32 ordinary ones."""
    cam = syn.config2(G=16, n_views=2)["cams"][1]
    rng = np.random.default_rng(7)
    n = 400000
    d = rng.uniform(0.2, 0.3, n)
    mc = np.stack([rng.uniform(-12, 12, n) * d, rng.uniform(-12, 12, n) * d, d], 1)
    means = ((mc - cam["t_v"].astype(np.float64)) @ cam["R_v"].astype(np.float64)).astype(np.float32)
    ls = np.stack([rng.normal(-8.5, 0.3, n), rng.normal(-8.5, 0.3, n), rng.normal(-1.9, 0.3, n)], 1).astype(np.float32)
    q = rng.standard_normal((n, 4)).astype(np.float32)
    mu, conic, depth, keep = project(R, dict(means3d=means, log_scales=ls, quats=q), cam)
    big = conic.abs().max(1).values.numpy() > 1e6
    sel = np.concatenate([np.nonzero(big)[0][:32], np.nonzero(~big)[0][:32]])
    np.savez_compressed(os.path.join(out, "geom_near_plane.npz"), means3d=means[sel], log_scales=ls[sel], quats=q[sel],
                        ref_mu2d=mu.numpy()[sel], ref_conic=conic.numpy()[sel], ref_depth=depth.numpy()[sel],
                        ref_keep=keep.numpy()[sel], ref_clamped=big[sel], **cam_arrays(cam))


def gen_loss(R, out):
    lm = R.loss_manual
    arrays = {}
    rng = np.random.default_rng(41)
    for name, (H, W, win) in {"l48x40": (48, 40, 11), "l64x64": (64, 64, 11), "l9x12": (9, 12, 9)}.items():
        x = rng.uniform(0, 1, (H, W, 3))
        y = rng.uniform(0, 1, (H, W, 3))
        g = lm.gauss_1d(win=win)
        Mh, Mw = lm.band_matrix(H, g), lm.band_matrix(W, g)
        Sx = torch.tensor(x).permute(2, 0, 1).contiguous()
        Sy = torch.tensor(y).permute(2, 0, 1).contiguous()
        loss, grad = lm.loss_manual(Sx, Sy, Mh, Mw)
        S, _ = lm.ssim_fwd(Sx, Sy, Mh, Mw)
        arrays.update({f"{name}__x": x, f"{name}__y": y, f"{name}__loss": np.float64(loss.item()),
                       f"{name}__ssim": np.float64(S.mean().item()),
                       f"{name}__grad": grad.permute(1, 2, 0).numpy()})
    np.savez_compressed(os.path.join(out, "loss.npz"), **arrays)


def gen_optim(R, syn, out):
    g = torch.Generator().manual_seed(3)
    params = [torch.randn(50, 3, generator=g).requires_grad_(True),
              torch.randn(50, generator=g).requires_grad_(True),
              torch.tensor(-3.0).requires_grad_(True)]
    init = [x.detach().clone().numpy() for x in params]
    lrs = [1.6e-4, 5e-2, 1e-2]
    opt = torch.optim.Adam([{"params": [x], "lr": lr} for x, lr in zip(params, lrs)])
    grads = []
    for _ in range(4):
        gs = [torch.randn(x.shape, generator=g) * 0.1 for x in params]
        for x, gg in zip(params, gs):
            x.grad = gg.clone()
        opt.step()
        grads.append([gg.numpy() for gg in gs])
    arrays = {f"p{i}_init": init[i] for i in range(3)}
    arrays.update({f"p{i}_final": params[i].detach().numpy() for i in range(3)})
    arrays.update({f"p{i}_m": opt.state[params[i]]["exp_avg"].numpy() for i in range(3)})
    arrays.update({f"p{i}_v": opt.state[params[i]]["exp_avg_sq"].numpy() for i in range(3)})
    arrays.update({f"p{i}_g{s}": grads[s][i] for i in range(3) for s in range(4)})
    arrays["lrs"] = np.array(lrs)

    # SGLD (spike/mcmc.py:25-34)
    sc = syn.config0(seed=8, G=300)
    p = sc["params"]
    op = p["opacity_raw"].copy()
    op[::3] = -6.0                                   # near-dead gaussians get noise
    m = _Model()
    m.means3d, m.log_scales, m.quats = t(p["means3d"]), t(p["log_scales"]), t(p["quats"])
    m.opacity_raw = t(op)
    torch.manual_seed(123)
    eps = torch.randn_like(m.means3d)
    torch.manual_seed(123)
    R.mcmc.add_sgld_noise(m, 5e-3, noise_lr=5e5)
    arrays.update(sgld_means3d=p["means3d"], sgld_log_scales=p["log_scales"], sgld_quats=p["quats"],
                  sgld_opacity_raw=op, sgld_eps=eps.numpy(), sgld_out=m.means3d.numpy())

    # relocate (spike/mcmc.py:41-71)
    sc = syn.config1(seed=9, G=400, res=64)
    p = sc["params"]
    op = p["opacity_raw"].copy()
    rng = np.random.default_rng(9)
    op[rng.random(op.size) < 0.12] = -8.0
    m = _Model()
    for k in ("means3d", "log_scales", "quats", "color_dc", "color_rest"):
        setattr(m, k, t(p[k]))
    m.opacity_sh = torch.zeros(op.size, 9)
    m.opacity_raw = t(op)
    torch.manual_seed(77)
    o = torch.sigmoid(m.opacity_raw)
    dead = torch.where(o < 0.005)[0]
    alive = torch.where(o >= 0.005)[0]
    probs = o[alive] / o[alive].sum()
    targets = alive[torch.multinomial(probs, dead.numel(), replacement=True)]
    noise = torch.stack([torch.randn(3) for _ in range(dead.numel())])
    torch.manual_seed(77)
    moved, touched = R.mcmc.relocate(m, dead_thr=0.005, offset=0.005)
    arrays.update({f"reloc_in_{k}": p[k] for k in ("means3d", "log_scales", "quats", "color_dc", "color_rest")})
    arrays.update(reloc_in_opacity_raw=op, reloc_targets=targets.numpy(), reloc_noise=noise.numpy(),
                  reloc_moved=moved, reloc_touched=touched.numpy())
    arrays.update({f"reloc_out_{k}": getattr(m, k).numpy() for k in
                   ("means3d", "log_scales", "quats", "color_dc", "color_rest", "opacity_raw")})
    np.savez_compressed(os.path.join(out, "optim.npz"), **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    R = import_reference(os.path.abspath(args.reference))
    syn = load_synthetic()
    torch.set_num_threads(os.cpu_count())
    jobs = dict(bins_scene=lambda: gen_bins_scene(R, syn, HERE), bins_stress=lambda: gen_bins_stress(R, syn, HERE),
                bins_radius=lambda: gen_bins_stress(R, syn, HERE, RADIUS_CASES, "bins_radius.npz"),
                bins_big=lambda: gen_bins_big(R, syn, HERE), render=lambda: gen_render(R, syn, HERE),
                geom=lambda: gen_geom(R, syn, HERE), loss=lambda: gen_loss(R, HERE),
                optim=lambda: gen_optim(R, syn, HERE), arm_b=lambda: gen_arm_b(R, syn, HERE),
                arm_rv=lambda: gen_arm_rv(R, syn, HERE), sh12=lambda: gen_sh12(R, syn, HERE),
                near_plane=lambda: gen_near_plane(R, syn, HERE))
    for name, fn in jobs.items():
        if args.only and name not in args.only.split(","):
            continue
        print("generating", name, flush=True)
        fn()


if __name__ == "__main__":
    main()
