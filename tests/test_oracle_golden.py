"""The oracle against the reference's own outputs (golden fixtures) and known answers.

CPU only.  Fixtures come from ``tests/golden/make_golden.py`` (the reference run in the build
container); known-answer values come from ``spike/tests/test_transform.py:15-31`` and
``spike/tests/test_toy_1g.py:21-57``.
"""
import numpy as np
import pytest

from conftest import cam_from, golden, params_from, rel_l2
from oracle import binning, geometry, loss as oloss, optim, pipeline, render, sh


def _check_tables(bins, idx_ref, valid_ref):
    assert np.array_equal(bins.valid, valid_ref)
    assert np.array_equal(np.where(bins.valid, bins.idx, -1), np.where(valid_ref, idx_ref, -1))


def test_bins_config0_bit_exact_vs_reference_stable():
    z = golden("bins_config0.npz")
    cam = cam_from(z)
    tm = binning.tile_map(cam["H"], cam["W"])
    b = binning.assign_bins(z["mu2d"], z["keep"], tm, int(z["R"]), int(z["K"]))
    _check_tables(b, z["idx_stable"], z["valid_stable"])
    assert np.array_equal(b.cand, z["cand"])


def test_bins_config0_unstable_reference_differs_only_inside_ties():
    """The unpatched reference uses a non-stable argsort: per tile the kept SET matches the
    canonical table except where the K boundary falls inside a run of equal keys."""
    z = golden("bins_config0.npz")
    cam = cam_from(z)
    tm = binning.tile_map(cam["H"], cam["W"])
    K = int(z["K"])
    b = binning.assign_bins(z["mu2d"], z["keep"], tm, 1, K)
    for t in range(tm.T):
        a = set(b.idx[t][b.valid[t]].tolist())
        r = set(z["idx_default"][t][z["valid_default"][t]].tolist())
        if a != r:
            assert b.cand[t] > K and b.q[t, K - 1] >= 0
            # the boundary key is shared with a dropped candidate (a tie)
            tiles, gs, js = binning.candidate_pairs(z["mu2d"], z["keep"], tm, 1)
            sel = tiles == t
            _, q = binning.quantised_dist2(z["mu2d"][gs[sel]], tiles[sel], tm.ntx)
            assert (q == b.q[t, K - 1]).sum() > 1


def test_bins_config1_digest_and_overflow():
    z = golden("bins_config1.npz")
    cam = cam_from(z)
    tm = binning.tile_map(cam["H"], cam["W"])
    b = binning.assign_bins(z["mu2d"], z["keep"], tm, 1, 128)
    assert np.array_equal(b.cand, z["cand"])
    assert int((b.count == 128).sum()) == int(z["full_tiles"]) > 0
    assert binning.table_digest(b) == str(z["digest"])


_MG = __import__("make_golden_cases")


@pytest.mark.parametrize("fixture,case", [("bins_stress.npz", c[0]) for c in _MG.STRESS_CASES]
                         + [("bins_radius.npz", c[0]) for c in _MG.RADIUS_CASES])
def test_bins_stress_bit_exact(fixture, case, pkg):
    name, seed, G, H, W, R, K, kw = next(c for c in _MG.STRESS_CASES + _MG.RADIUS_CASES if c[0] == case)
    z = golden(fixture)
    mu, keep = pkg.synthetic.stress_mu2d(seed, G, H, W, **kw)
    tm = binning.tile_map(H, W)
    b = binning.assign_bins(mu, keep, tm, R, K)
    _check_tables(b, z[f"{name}__idx_stable"], z[f"{name}__valid_stable"])
    assert np.array_equal(b.cand, z[f"{name}__cand"])


def test_bins_big_digest(pkg):
    import hashlib
    import make_golden_cases as mg
    c = mg.BIG_CASE
    z = golden("bins_big.npz")
    mu, keep = pkg.synthetic.stress_mu2d(c["seed"], c["G"], c["H"], c["W"], **c["kw"])
    assert hashlib.sha256(mu.tobytes()).hexdigest() == str(z["mu_sha"])
    tm = binning.tile_map(c["H"], c["W"])
    b = binning.assign_bins(mu, keep, tm, c["R"], c["K"])
    assert np.array_equal(b.cand, z["cand"])
    assert int(np.maximum(b.cand - c["K"], 0).sum()) == int(z["overflow"])
    assert binning.table_digest(b) == str(z["digest"])


def test_inverse_table_matches_build_inv():
    z = golden("bins_config0.npz")
    cam = cam_from(z)
    tm = binning.tile_map(cam["H"], cam["W"])
    b = binning.assign_bins(z["mu2d"], z["keep"], tm, 1, 128)
    G = z["mu2d"].shape[0]
    ref = binning.build_inv(b.idx, b.valid, G, 9)
    mine = binning.stencil_inv(b, G, 1)
    TK = b.idx.size
    for g in range(G):
        assert set(ref[g][ref[g] != TK].tolist()) == set(mine[g][mine[g] >= 0].tolist())
    grad = np.random.default_rng(0).standard_normal((tm.T, 128, 9))
    grad *= b.valid[..., None]
    pad = np.where(mine >= 0, mine, TK)
    a = binning.gather_reduce(grad, pad)
    r = np.zeros((G, 9))
    np.add.at(r, b.idx.reshape(-1), grad.reshape(-1, 9))
    assert np.abs(a - r).max() < 1e-9


def test_theta_known_answer():
    """spike/tests/test_transform.py:15-31: conic (0.08,0.02,0.05), mu (3.5,4.5), k=4."""
    th = render.theta_u_gathered(np.array([[[0.08, 0.02, 0.05]]]), np.array([[[3.5, 4.5]]]),
                                 np.zeros((1, 2)), 4.0)[0, :, 0].astype(np.float64)
    theta_Q = np.array([0.08, 0.05, 0.04, -0.74, -0.59, 2.6225])
    assert np.allclose(th, -theta_Q / 4 + np.array([0, 0, 0, 0, 0, 1.0]), atol=1e-6)
    phi = np.array([25.0, 36.0, 30.0, 5.0, 6.0, 1.0])
    assert abs(phi @ th - 0.904375) < 1e-6
    assert abs(phi @ theta_Q - 0.3825) < 1e-9


def test_toy_single_gaussian():
    """spike/tests/test_toy_1g.py:21-57: centre pixel -> the colour, cutoff -> background."""
    conic = np.array([[0.25, 0.0, 0.25]])
    mu = np.array([[8.0, 8.0]])
    th = render.theta_u_gathered(conic[None], mu[None], np.zeros((1, 2)), 4.0)[0].T   # [1,6]
    color = np.array([[0.7, 0.2, 0.1]])
    Phi = np.array([[64.0, 64.0, 64.0, 8.0, 8.0, 1.0], [144.0, 64.0, 96.0, 12.0, 8.0, 1.0]])
    C = render.wsr_dense_fwd(th, np.array([0.8]), color, 1e-6, Phi, np.ones(3))
    assert np.allclose(C[0], color[0], atol=1e-3)
    assert np.allclose(C[1], 1.0, atol=1e-3)


def test_render_config0_vs_reference():
    z = golden("render_config0.npz")
    cam = cam_from(z)
    p = params_from(z)
    tm = binning.tile_map(cam["H"], cam["W"])
    fw = pipeline.render_view(p, 0, cam, K=int(z["K"]))
    # same tables as the reference on the reference's own mu2d
    assert np.array_equal(np.where(fw["bins"].valid, fw["bins"].idx, -1), np.where(z["valid"], z["idx"], -1))
    assert (np.abs(fw["theta"] - z["theta_u"]) <= 1e-4 * np.maximum(1.0, np.abs(z["theta_u"]))).all()
    assert np.abs(fw["img"] - z["img"]).max() < 1e-4          # geometry evaluated in float64
    # binned forward on the reference's operands is (nearly) bit-exact
    img, den, _ = render.render_fwd(z["theta_u"], z["col"], z["oc"], z["w_b"], np.ones(3, np.float32), tm)
    assert np.abs(img - z["img"]).max() < 2e-6
    assert np.abs(den - z["den"]).max() < 2e-5 * np.abs(z["den"]).max()


def test_render_backward_config0_vs_reference_autograd():
    z = golden("render_config0.npz")
    cam = cam_from(z)
    tm = binning.tile_map(cam["H"], cam["W"])
    img = z["img"]
    N = img.size
    gimg = (np.sign(img - z["target"]) / N).astype(np.float32)
    gth, gcol, goc, gwb = render.render_bwd(gimg, z["theta_u"], z["col"], z["oc"], z["w_b"],
                                            np.ones(3, np.float32), tm)
    assert rel_l2(gth, z["gtheta"]) < 1e-5
    assert rel_l2(gcol, z["gcol"]) < 1e-5
    assert rel_l2(goc, z["goc"]) < 1e-5
    assert abs(gwb - z["gw_b"]) < 1e-5 * abs(z["gw_b"]) + 1e-9


@pytest.mark.parametrize("fixture,deg", [("render_config0.npz", 0), ("render_sh3.npz", 3)])
def test_param_grads_vs_reference_autograd(fixture, deg):
    z = golden(fixture)
    cam = cam_from(z)
    p = params_from(z)
    fw = pipeline.render_view(p, deg, cam, K=int(z["K"]))
    assert np.array_equal(np.where(fw["bins"].valid, fw["bins"].idx, -1), np.where(z["valid"], z["idx"], -1))
    assert np.abs(fw["img"] - z["img"]).max() < 1e-4
    N = fw["img"].size
    gimg = (np.sign(fw["img"] - z["target"]) / N).astype(np.float32)
    g = pipeline.backward_view(fw, gimg, p, deg)
    names = ["means3d", "log_scales", "quats", "opacity_raw", "color_dc"] + (["color_rest"] if deg else [])
    for n in names:
        assert rel_l2(g[n], z["grad_" + n]) < 1e-3, (n, rel_l2(g[n], z["grad_" + n]))
    assert abs(g["w_b_raw"] - float(z["grad_w_b_raw"])) < 1e-3 * abs(float(z["grad_w_b_raw"]))


@pytest.mark.parametrize("deg", [0, 3])
def test_arm_b_vs_reference_autograd(deg):
    """Arm B (opacity x sigmoid(depth_beta (depth_tau - z))) image and gradients, including the
    two depth parameters, against the reference's dense render + autograd."""
    z = golden("render_arm_b.npz")
    cam = cam_from(z)
    p = params_from(z)
    bt = (float(z["depth_beta"]), float(z["depth_tau"]))
    fw = pipeline.render_view(p, deg, cam, K=int(z["K"]), depth_bt=bt)
    pre = f"deg{deg}__"
    assert np.abs(fw["img"] - z[pre + "img"]).max() < 1e-4
    g = pipeline.backward_view(fw, z["wts"].astype(np.float32), p, deg)
    names = ["means3d", "log_scales", "quats", "opacity_raw", "color_dc"] + (["color_rest"] if deg else [])
    for n in names:
        assert rel_l2(g[n], z[pre + "grad_" + n]) < 1e-3, (n, rel_l2(g[n], z[pre + "grad_" + n]))
    for n in ("w_b_raw", "depth_beta", "depth_tau"):
        ref = float(z[pre + "grad_" + n])
        assert abs(g[n] - ref) < 1e-3 * abs(ref), (n, g[n], ref)


@pytest.mark.parametrize("deg", [0, 3])
def test_arm_rv_vs_reference_autograd(deg):
    """Arm RV (revealage compositing) image and gradients against the reference's dense render +
    autograd; the fixture has pixel weights above the clamp bound (no gradient there)."""
    z = golden("render_arm_rv.npz")
    cam = cam_from(z)
    p = params_from(z)
    fw = pipeline.render_view(p, deg, cam, K=int(z["K"]), arm="RV")
    assert (fw["rcache"][2] > render.RV_AMAX).any()
    pre = f"deg{deg}__"
    assert np.abs(fw["img"] - z[pre + "img"]).max() < 1e-4
    g = pipeline.backward_view(fw, z["wts"].astype(np.float32), p, deg)
    names = ["means3d", "log_scales", "quats", "opacity_raw", "color_dc"] + (["color_rest"] if deg else [])
    for n in names:
        assert rel_l2(g[n], z[pre + "grad_" + n]) < 1e-3, (n, rel_l2(g[n], z[pre + "grad_" + n]))
    assert g["w_b_raw"] == 0.0


@pytest.mark.parametrize("deg", [1, 2])
def test_sh_degree_1_2_vs_reference_autograd(deg):
    """Arm A at SH degrees 1 and 2 (the degrees between DC-only and the full 16 coefficients)."""
    z = golden("render_sh12.npz")
    cam = cam_from(z)
    p = params_from(z)
    fw = pipeline.render_view(p, deg, cam, K=int(z["K"]))
    pre = f"deg{deg}__"
    assert np.abs(fw["img"] - z[pre + "img"]).max() < 1e-4
    g = pipeline.backward_view(fw, z["wts"].astype(np.float32), p, deg)
    for n in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest"):
        assert rel_l2(g[n], z[pre + "grad_" + n]) < 1e-3, (n, rel_l2(g[n], z[pre + "grad_" + n]))
    ref = float(z[pre + "grad_w_b_raw"])
    assert abs(g["w_b_raw"] - ref) < 1e-3 * abs(ref)


def test_geometry_bwd_vs_reference():
    z = golden("geom_bwd.npz")
    cam = cam_from(z)
    conic, mu2d, _, _, cache = geometry.fwd(z["means3d"], z["quats"], z["log_scales"], cam)
    assert rel_l2(conic, z["conic"]) < 1e-5 and rel_l2(mu2d, z["mu2d"]) < 1e-6
    gc, gm = z["gconic"].astype(np.float64), z["gmu"].astype(np.float64)
    gmeans, gq, gs = geometry.bwd(cache, gc[:, 0], gc[:, 1], gc[:, 2], gm[:, 0], gm[:, 1])
    assert rel_l2(gmeans, z["gmeans"]) < 1e-4
    assert rel_l2(gq, z["gquats"]) < 1e-4
    assert rel_l2(gs * cache["scale"], z["glog_scales"]) < 1e-4
    # the dense project_ewa agrees with the per-component form
    R = geometry.quat_to_rotmat(z["quats"])
    mu_d, conic_d, _, _ = geometry.project_ewa(z["means3d"], geometry.cov3d(np.exp(z["log_scales"].astype(np.float64)), R),
                                               cam["R_v"], cam["t_v"], cam["fx"], cam["fy"], cam["cx"], cam["cy"])
    assert rel_l2(conic_d, conic) < 1e-12 and rel_l2(mu_d, mu2d) < 1e-12


def test_near_plane_needles_reference_fp32_clamps_where_float64_is_bounded():
    """Thin gaussians just past the near plane, projecting far off-screen (fixture written by the
    reference's fp32 project_ewa, spike/geometry.py:28-57): for half of them the reference's
    det = s00 s11 - s01^2 cancels to noise and its 1e-12 clamp yields conics of ~1e20, while in
    float64 every conic is positive definite and bounded by 1/blur (det(J S J^T + blur I) >=
    blur^2).  The oracle keeps the float64 values, which the device's fused projection matches
    (tests/test_gpu_render.py)."""
    z = golden("geom_near_plane.npz")
    cam = cam_from(z)
    conic, mu2d, depth, keep, _ = geometry.fwd(z["means3d"], z["quats"], z["log_scales"], cam)
    clamped = z["ref_clamped"]
    assert clamped.sum() >= 16 and (~clamped).sum() >= 16
    assert np.abs(z["ref_conic"][clamped]).max(1).min() > 1e6
    assert keep.all() and z["ref_keep"].all()
    assert np.abs(conic).max() <= 1.0 / 0.3 + 1e-9
    assert (conic[:, 0] > 0).all() and (conic[:, 0] * conic[:, 2] - conic[:, 1] ** 2 > 0).all()
    # the means are well conditioned in fp32; the conics of these needles are not (even where the
    # reference's clamp did not fire, its fp32 conic is off by up to order one)
    assert np.abs(z["ref_mu2d"] - mu2d).max() / np.abs(mu2d).max() < 1e-5


def test_geometry_analytic_isotropic():
    """spike/tests/test_geometry_analytic.py:12-35."""
    cam = dict(R_v=np.eye(3), t_v=np.array([0.0, 0.0, 4.0]), fx=178.0, fy=178.0, cx=64.0, cy=64.0)
    s = 0.1
    conic, mu2d, depth, keep, _ = geometry.fwd(np.zeros((1, 3)), np.array([[1.0, 0, 0, 0]]),
                                               np.log(np.full((1, 3), s)), cam)
    pred = 1.0 / ((s * 178.0 / 4.0) ** 2 + 0.3)
    assert np.allclose(mu2d[0], [64.0, 64.0]) and keep[0]
    assert abs(conic[0, 0] - pred) < 1e-9 and abs(conic[0, 2] - pred) < 1e-9 and abs(conic[0, 1]) < 1e-12


def test_sh_backward_finite_difference():
    rng = np.random.default_rng(2)
    coeffs = rng.standard_normal((6, 16, 3))
    dirs = rng.standard_normal((6, 3))
    gcol = rng.standard_normal((6, 3))
    gco, gd = sh.eval_sh_color_bwd(3, coeffs, dirs, gcol)

    def f(c, d):
        return (sh.eval_sh_color(3, c, d)[0] * gcol).sum()
    eps = 1e-6
    for _ in range(10):
        i, k, ch = rng.integers(6), rng.integers(16), rng.integers(3)
        c2 = coeffs.copy(); c2[i, k, ch] += eps
        c1 = coeffs.copy(); c1[i, k, ch] -= eps
        assert abs((f(c2, dirs) - f(c1, dirs)) / (2 * eps) - gco[i, k, ch]) < 1e-6
        j = rng.integers(3)
        d2 = dirs.copy(); d2[i, j] += eps
        d1 = dirs.copy(); d1[i, j] -= eps
        assert abs((f(coeffs, d2) - f(coeffs, d1)) / (2 * eps) - gd[i, j]) < 1e-5


def test_sh_zero_rest_equals_dc():
    """spike/tests/test_sh_color.py:22-29."""
    rng = np.random.default_rng(0)
    dc = rng.standard_normal((50, 3))
    coeffs = np.concatenate([dc[:, None], np.zeros((50, 15, 3))], 1)
    for deg in range(4):
        c, _ = sh.eval_sh_color(deg, coeffs, rng.standard_normal((50, 3)))
        assert np.allclose(c, np.maximum(0.5 + sh.C0 * dc, 0.0), atol=1e-12)


@pytest.mark.parametrize("case", ["l48x40", "l64x64", "l9x12"])
def test_loss_vs_reference_restatement(case):
    z = golden("loss.npz")
    x, y = z[f"{case}__x"], z[f"{case}__y"]
    loss, ssim, _, grad = oloss.loss_and_grad(x, y, 0.2)
    assert abs(ssim - float(z[f"{case}__ssim"])) < 1e-12
    assert abs(loss - float(z[f"{case}__loss"])) < 1e-12
    assert rel_l2(grad, z[f"{case}__grad"]) < 1e-10


def _ssim_published(pred, gt, win_size=11):
    """SSIM as pytorch_msssim 1.0.0 publishes it, restated independently of the oracle, for
    spike/metrics.py:15-19's call ssim(clamp(pred), clamp(gt), data_range=1, win_size=w): a
    normalised 1-D Gaussian of sigma 1.5 over arange(w) - w // 2, applied without padding along
    H then along W (scipy correlation, mode "valid"), K = (0.01, 0.03), the map
    ((2 mu1 mu2 + C1) / (mu1^2 + mu2^2 + C1)) * ((2 s12 + C2) / (s1^2 + s2^2 + C2)) averaged per
    channel, then over the channels."""
    from scipy.signal import correlate
    H, W = pred.shape[:2]
    w = min(win_size, H, W)
    w = max(w - 1 if w % 2 == 0 else w, 3)
    c = np.arange(w, dtype=np.float64) - w // 2
    g = np.exp(-(c ** 2) / (2 * 1.5 ** 2))
    g = g / g.sum()

    def blur(m):
        return correlate(correlate(m, g[:, None], mode="valid"), g[None, :], mode="valid")

    C1, C2 = 0.01 ** 2, 0.03 ** 2
    per_channel = []
    for ch in range(3):
        X = np.clip(np.asarray(pred[..., ch], np.float64), 0.0, 1.0)
        Y = np.clip(np.asarray(gt[..., ch], np.float64), 0.0, 1.0)
        mu1, mu2 = blur(X), blur(Y)
        s1 = blur(X * X) - mu1 * mu1
        s2 = blur(Y * Y) - mu2 * mu2
        s12 = blur(X * Y) - mu1 * mu2
        cs = (2 * s12 + C2) / (s1 + s2 + C2)
        per_channel.append((((2 * mu1 * mu2 + C1) / (mu1 * mu1 + mu2 * mu2 + C1)) * cs).mean())
    return float(np.mean(per_channel))


@pytest.mark.parametrize("shape", [(40, 56), (17, 23), (8, 12), (6, 6)])
def test_oracle_ssim_equals_the_published_algorithm(shape):
    """The oracle's SSIM (restated from tools/loss_manual.py) equals an independent restatement
    of pytorch_msssim's published algorithm, including the shrunken odd window of small images
    and the [0, 1] clamp of the inputs; the loss then follows as (1 - l) L1 + l (1 - SSIM)."""
    rng = np.random.default_rng(sum(shape))
    pred = rng.uniform(-0.2, 1.2, shape + (3,))
    gt = rng.uniform(0.0, 1.0, shape + (3,))
    loss, ssim, l1, _ = oloss.loss_and_grad(pred, gt, 0.2)
    ref = _ssim_published(pred, gt)
    assert abs(ssim - ref) < 1e-12, (ssim, ref)
    assert abs(loss - (0.8 * np.abs(pred - gt).mean() + 0.2 * (1.0 - ref))) < 1e-12


def test_loss_clamp_gradient_finite_difference():
    rng = np.random.default_rng(5)
    x = rng.uniform(-0.3, 1.3, (20, 22, 3))
    y = rng.uniform(0, 1, (20, 22, 3))
    _, _, _, g = oloss.loss_and_grad(x, y)
    eps = 1e-7
    for _ in range(12):
        i, j, c = rng.integers(20), rng.integers(22), rng.integers(3)
        if min(abs(x[i, j, c]), abs(x[i, j, c] - 1), abs(x[i, j, c] - y[i, j, c])) < 1e-5:
            continue
        xp = x.copy(); xp[i, j, c] += eps
        xm = x.copy(); xm[i, j, c] -= eps
        fd = (oloss.loss_and_grad(xp, y)[0] - oloss.loss_and_grad(xm, y)[0]) / (2 * eps)
        assert abs(fd - g[i, j, c]) < 1e-6 * max(1.0, abs(fd)) + 1e-9


def test_adam_vs_torch_reference():
    z = golden("optim.npz")
    lrs = z["lrs"]
    for i in range(3):
        p = np.atleast_1d(z[f"p{i}_init"]).astype(np.float32).copy()
        m = np.zeros_like(p)
        v = np.zeros_like(p)
        for s in range(4):
            optim.adam_update(p, np.atleast_1d(z[f"p{i}_g{s}"]).astype(np.float32), m, v, s + 1, float(lrs[i]))
        assert np.abs(p - np.atleast_1d(z[f"p{i}_final"])).max() < 1e-6
        assert np.abs(m - np.atleast_1d(z[f"p{i}_m"])).max() < 1e-7


def test_sgld_vs_reference():
    z = golden("optim.npz")
    out = optim.sgld_noise(z["sgld_means3d"], z["sgld_log_scales"], z["sgld_quats"], z["sgld_opacity_raw"],
                           z["sgld_eps"], 5e-3, 5e5)
    assert (np.abs(out - z["sgld_out"]) <= 1e-5 * np.maximum(1.0, np.abs(z["sgld_out"]))).all()
    moved = np.abs(z["sgld_out"] - z["sgld_means3d"]).max(1)
    assert moved[::3].min() > 0        # near-dead gaussians received noise


def test_relocate_vs_reference():
    z = golden("optim.npz")
    p = {k: z[f"reloc_in_{k}"].astype(np.float32).copy() for k in
         ("means3d", "log_scales", "quats", "color_dc", "color_rest", "opacity_raw")}
    moved, touched = optim.relocate(p, 0.005, z["reloc_targets"], z["reloc_noise"], offset=0.005)
    assert moved == int(z["reloc_moved"]) > 0
    assert np.array_equal(touched, z["reloc_touched"])
    for k in p:
        assert np.abs(p[k] - z[f"reloc_out_{k}"]).max() < 1e-6, k


def _bf16(x):
    """Round float32 to bfloat16 (nearest, ties to even) and back, by the bit pattern."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def test_tile_local_theta_matches_global_quad_form():
    """spike/tests/test_tile_local.py:22-38 on the oracle's theta_u_gathered: with the tile origin
    folded into theta, Phi.theta (k = 1) gives 1 - Q of the global quadratic form at every pixel
    centre of the tile, to float32 rounding (the operand build is float32, as in the reference)."""
    from oracle.render import theta_u_gathered
    rng = np.random.default_rng(1)
    Phi = binning.tile_map(16, 16).Phi.astype(np.float64)
    lx, ly = Phi[:, 3], Phi[:, 4]
    for _ in range(20):
        origin = rng.integers(0, 64, 2).astype(np.float64) * 16.0
        L = rng.standard_normal((5, 2, 2))
        M = L @ np.transpose(L, (0, 2, 1)) + 0.1 * np.eye(2)
        conic = np.stack([M[:, 0, 0], M[:, 0, 1], M[:, 1, 1]], -1)
        mu = origin + rng.random((5, 2)) * 16.0
        th = theta_u_gathered(conic[None], mu[None], origin[None], 1.0)[0].astype(np.float64)   # [6, G]
        q_local = 1.0 - Phi @ th
        dx = (origin[0] + lx)[:, None] - mu[None, :, 0].astype(np.float32)
        dy = (origin[1] + ly)[:, None] - mu[None, :, 1].astype(np.float32)
        a, b, c = (conic[:, i].astype(np.float32) for i in range(3))
        q_global = a * dx * dx + 2 * b * dx * dy + c * dy * dy
        scale = np.abs(th).max(0) * 256.0 + 1.0      # largest monomial term per gaussian
        assert (np.abs(q_local - q_global) <= 1e-7 * scale).all()


def test_tile_local_theta_survives_bf16():
    """spike/tests/test_tile_local.py:41-70: in bfloat16 the tile-local Phi.theta keeps Q within
    0.1 of the float64 value, while the same product in global pixel coordinates loses it."""
    from oracle.render import theta_u_gathered
    origin = np.array([400.0, 400.0])
    conic = np.array([[0.08, 0.02, 0.05]])
    mu = origin + np.array([[7.3, 4.6]])
    Phi = binning.tile_map(16, 16).Phi
    px, py = origin[0] + Phi[:, 3].astype(np.float64), origin[1] + Phi[:, 4].astype(np.float64)
    dx, dy = px - mu[0, 0], py - mu[0, 1]
    q_ref = 0.08 * dx * dx + 2 * 0.02 * dx * dy + 0.05 * dy * dy
    th_local = theta_u_gathered(conic[None], mu[None], origin[None], 1.0)[0]
    q_local = 1.0 - (_bf16(Phi).astype(np.float64) @ _bf16(th_local).astype(np.float64))[:, 0]
    th_global = theta_u_gathered(conic[None], mu[None], np.zeros((1, 2)), 1.0)[0]
    Phi_g = np.stack([px * px, py * py, px * py, px, py, np.ones_like(px)], -1).astype(np.float32)
    q_global = 1.0 - (_bf16(Phi_g).astype(np.float64) @ _bf16(th_global).astype(np.float64))[:, 0]
    err_local = np.abs(q_local - q_ref).max()
    err_global = np.abs(q_global - q_ref).max()
    assert err_local < 0.1
    assert err_global > 1.0 and err_global > 20 * err_local
