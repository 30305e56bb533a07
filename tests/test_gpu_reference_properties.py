"""The reference's own property tests, run on the device path.

Each test restates one of ``spike/tests``' claims about the renderer and the optimiser and checks
it through the CUDA kernels (binned render, train step, device SGLD and relocation) instead of
the reference's CPU torch code:

- ``test_mcmc.py:24-51``: n coincident copies at opacity o/n render like one gaussian at o under
  the weighted-sum (WSR) blend, and a wrong split (copies kept at o) does not (negative control);
- ``test_mcmc.py:54-65``: relocating near-dead gaussians onto live ones leaves the render almost
  unchanged;
- ``test_mcmc.py:68-77``: the SGLD noise is gated by opacity (a settled gaussian does not move);
- ``test_synthetic_overfit.py:11-19``: every arm renders finite, bounded images;
- ``test_synthetic_overfit.py:30-44``: a fresh model fitted to the renders of a known scene
  recovers it (loss below 0.3x its start, PSNR up by 8 dB and above 24 dB);
- ``test_toy_occlusion.py:44-48``: the depth-free arm A averages two gaussians at the same place;
- ``test_geometry_analytic.py:12-61``: the EWA projection of an isotropic gaussian is analytic,
  scales with depth, and culls at the near plane;
- ``test_toy_1g.py:21-60``: a single gaussian's closed-form centre, cutoff and beyond-cutoff pixels.

Image sizes are the reference's rounded up to whole 16-pixel tiles (the binned path's tiling):
24 -> 32 and 40 -> 48.  The oracle reaches 44.9 dB on the overfit case at 48x48 (400 steps).
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _logit(p):
    return math.log(p / (1.0 - p))


def _orbit_cameras(n, res, radius=2.5, elevation=0.6, fov=0.7):
    """Cameras on a ring around the origin looking at it (spike/synthetic.py:20-30's layout)."""
    from tt_splat_b200 import camera
    f = 0.5 * res / math.tan(0.5 * fov)
    cams = []
    for i in range(n):
        th = 2.0 * math.pi * i / n
        R_v, t_v = camera.look_at_opencv((radius * math.cos(th), elevation, radius * math.sin(th)), (0.0, 0.0, 0.0))
        cams.append(camera.Camera(R_v, t_v, f, f, res / 2.0, res / 2.0, res, res))
    return cams


def test_opacity_split_preserves_render():
    """n copies of one gaussian at o/n render like the gaussian at o; copies left at o do not."""
    from tt_splat_b200 import model, render
    cam = _orbit_cameras(1, 32)[0]
    o0, n = 0.6, 4
    base = model.GaussianModel(n, seed=3, device=DEV)
    with torch.no_grad():
        for name in ("log_scales", "quats", "color_dc"):
            t = getattr(base, name)
            t[:] = t[0:1].clone()
        base.means3d[:] = 0.0                        # on the optical axis, so it covers pixels
        base.log_scales[:] = math.log(0.15)
        base.opacity_raw[:] = _logit(o0 / n)
    single = model.GaussianModel(1, seed=3, device=DEV)
    with torch.no_grad():
        for name in ("means3d", "log_scales", "quats", "color_dc"):
            getattr(single, name)[:] = getattr(base, name)[0:1]
        single.w_b_raw.copy_(base.w_b_raw)
        single.opacity_raw[:] = _logit(o0)
        C_multi = render.render(base, cam)
        C_single = render.render(single, cam)
        assert (C_single - C_multi).abs().max().item() < 1e-5
        base.opacity_raw[:] = _logit(o0)             # negative control: the wrong split
        C_wrong = render.render(base, cam)
    assert (C_wrong - C_single).abs().max().item() > 1e-3, "the test does not discriminate"


def test_relocation_keeps_render():
    """Relocating 12 near-dead gaussians (opacity 1e-4) onto live ones by the o/n split changes
    the image by what the dead ones contributed (the oracle: 2.0e-3 for any draw)."""
    from tt_splat_b200 import mcmc, model, render
    cam = _orbit_cameras(1, 32)[0]
    m = model.GaussianModel(40, extent=0.6, seed=5, gt=True, device=DEV)
    with torch.no_grad():
        m.opacity_raw[:12] = _logit(1e-4)
        before = render.render(m, cam)
    moved, touched = mcmc.relocate(m, dead_thr=0.005, offset=0.0)
    with torch.no_grad():
        after = render.render(m, cam)
    assert moved == 12, moved
    assert touched.numel() > 0
    assert (before - after).abs().max().item() < 2e-2
    assert bool((torch.sigmoid(m.opacity_raw) >= 0.005).all())       # no dead gaussian left


def test_sgld_noise_is_opacity_gated():
    from tt_splat_b200 import mcmc, model
    m = model.GaussianModel(2, seed=1, device=DEV)
    with torch.no_grad():
        m.opacity_raw[0] = _logit(0.99)              # settled: no noise
        m.opacity_raw[1] = _logit(1e-3)              # near-dead: noise
    before = m.means3d.detach().clone()
    mcmc.add_sgld_noise(m, lr=5e-3, noise_lr=100.0)
    disp = (m.means3d.detach() - before).norm(dim=1)
    assert disp[0].item() < 1e-6, disp[0].item()
    assert disp[1].item() > disp[0].item()


@pytest.mark.parametrize("arm", ["A", "B", "RV"])
def test_render_arms_finite(arm):
    from tt_splat_b200 import model, render
    gt = model.GaussianModel(30, extent=0.5, seed=1, gt=True, init_scale=0.08, device=DEV)
    cam = _orbit_cameras(1, 32)[0]
    with torch.no_grad():
        img = render.render(gt, cam, arm)
    assert tuple(img.shape) == (32, 32, 3)
    assert bool(torch.isfinite(img).all())
    assert img.min().item() >= -1e-4 and img.max().item() < 5.0


def test_overfit_recovers():
    """The reference's data-free self-consistency oracle: render a known 30-gaussian scene from 4
    views, fit a fresh 150-gaussian model to the renders for 400 Adam steps through the train
    step, and recover the images."""
    from tt_splat_b200 import model, render, train
    gt = model.GaussianModel(30, extent=0.5, seed=1, gt=True, init_scale=0.08, device=DEV)
    cams = _orbit_cameras(4, 48)
    with torch.no_grad():
        imgs = [render.render(gt, c).detach().clone() for c in cams]
    m = model.GaussianModel(150, extent=0.7, seed=2, gt=False, device=DEV)
    psnr0 = train.eval_psnr(m, cams, imgs)
    hist = train.fit(m, cams, imgs, iters=400)
    psnr1 = train.eval_psnr(m, cams, imgs)
    assert hist[-1] < 0.3 * hist[0], (hist[0], hist[-1])
    assert psnr1 > psnr0 + 8.0, (psnr0, psnr1)
    assert psnr1 > 24.0, psnr1


def test_arm_a_averages_coincident_gaussians():
    """Two gaussians at one screen position with equal footprints, red and blue at opacity 0.9:
    the depth-free weighted sum shows their average (it does not model occlusion)."""
    from tt_splat_b200 import backward, forward
    f = lambda x: torch.tensor(x, dtype=torch.float32, device=DEV)  # noqa: E731
    mu2d = f([[0.0, 0.0], [0.0, 0.0]])
    conic = f([[0.25, 0.0, 0.25], [0.25, 0.0, 0.25]])
    red, blue = f([1.0, 0.0, 0.0]), f([0.0, 0.0, 1.0])
    px, py = f([0.0]), f([0.0])
    w_geo = forward.poly_splat_wgeo(forward.quad_form(px, py, mu2d, conic), 4.0)
    assert torch.allclose(w_geo, torch.ones_like(w_geo))
    _, theta_u = forward.theta_from_conic(conic, mu2d, 4.0)
    o = torch.sigmoid(f([_logit(0.9), _logit(0.9)]))
    C = backward.wsr_polysplat(theta_u, o, torch.stack([red, blue]), 1e-6, forward.phi(px, py), f([1.0, 1.0, 1.0]))[0]
    assert torch.allclose(C, 0.5 * (red + blue), atol=1e-3), C


def _iso_projection(z, s, blur, near=0.2, fx=178.0, cx=64.0):
    """One isotropic gaussian of world std s on the optical axis at depth z, float64."""
    from tt_splat_b200 import geometry
    d = dict(dtype=torch.float64, device=DEV)
    means = torch.zeros(1, 3, **d)
    cov = (s * s) * torch.eye(3, **d).unsqueeze(0)
    R_v = torch.eye(3, dtype=torch.float64)
    t_v = torch.tensor([0.0, 0.0, z], dtype=torch.float64)
    return geometry.project_ewa(means, cov, R_v, t_v, fx, fx, cx, cx, blur_eps=blur, near=near)


def test_isotropic_projection_is_analytic():
    """spike/tests/test_geometry_analytic.py:12-35 on the device kernel: the mean lands on the
    principal point and the conic diagonal is 1 / ((s fx / z)^2 + blur)."""
    s, z, fx, cx, blur = 0.1, 4.0, 178.0, 64.0, 0.3
    mu2d, conic, depth, keep = _iso_projection(z, s, blur)
    assert torch.allclose(mu2d[0].cpu(), torch.tensor([cx, cx], dtype=torch.float64), atol=1e-9)
    assert abs(depth.item() - z) < 1e-9 and bool(keep[0])
    pred = 1.0 / ((s * fx / z) ** 2 + blur)
    a, b, c = conic[0].tolist()
    assert abs(a - pred) < 1e-6 and abs(c - pred) < 1e-6, (a, c, pred)
    assert abs(b) < 1e-9


def test_projection_depth_scaling_and_near_cull():
    """spike/tests/test_geometry_analytic.py:38-61: twice the depth, four times the conic
    diagonal (no blur); a gaussian nearer than the near plane is not kept."""
    a8 = _iso_projection(8.0, 0.05, 0.0)[1][0, 0].item()
    a4 = _iso_projection(4.0, 0.05, 0.0)[1][0, 0].item()
    assert abs(a8 / a4 - 4.0) < 1e-6
    keep = _iso_projection(0.05, 0.1, 0.3, fx=100.0)[3]
    assert not bool(keep[0])


def test_single_gaussian_closed_form():
    """spike/tests/test_toy_1g.py:21-60 on the device primitives: at the centre Q = 0 and the
    pixel shows the gaussian's colour; at the cutoff radius Q = k, the weight is 0 and the pixel
    shows the background; beyond it the weight stays 0."""
    from tt_splat_b200 import backward, forward
    f = lambda x: torch.tensor(x, dtype=torch.float64, device=DEV)  # noqa: E731
    k, cx = 4.0, 8.0
    mu2d, conic = f([[cx, cx]]), f([[0.25, 0.0, 0.25]])
    color, c_b = f([[0.7, 0.2, 0.1]]), f([1.0, 1.0, 1.0])
    o = f([0.8])
    px, py = f([cx, cx + 4.0, cx + 10.0]), f([cx, cx, cx])
    Q = forward.quad_form(px, py, mu2d, conic)[:, 0]
    assert abs(Q[0].item()) < 1e-12 and abs(Q[1].item() - 4.0) < 1e-9 and Q[2].item() > k
    w = forward.poly_splat_wgeo(forward.quad_form(px, py, mu2d, conic), k)[:, 0]
    assert abs(w[0].item() - 1.0) < 1e-12 and w[1].item() == 0.0 and w[2].item() == 0.0
    _, theta_u = forward.theta_from_conic(conic, mu2d, k)
    C = backward.wsr_polysplat(theta_u, o, color, 1e-6, forward.phi(px, py), c_b)
    assert torch.allclose(C[0].double(), color[0], atol=1e-3), C[0]
    assert torch.allclose(C[1].double(), c_b, atol=1e-3), C[1]
