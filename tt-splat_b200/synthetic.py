"""Seeded synthetic scenes for the five benchmark configurations, and the reference's data-free
self-consistency scene (``make_scene`` and its parts, ``spike/synthetic.py``).

The reference measures on synthetic scenes only (no dataset ships with it), so every
scene here is drawn from a seeded ``numpy.random.Generator(PCG64)`` in float32.  The
draws are host-side and bit-reproducible on any machine with the same numpy, which is
what lets the test fixtures pin results by seed.

Parameter layout follows ``spike/model.py:16-51`` (GaussianModel): means3d[G,3],
log_scales[G,3], quats[G,4] (w,x,y,z), opacity_raw[G], color_dc[G,3],
color_rest[G,15,3], w_b_raw (scalar, -3 at init, ``spike/model.py:47``).  Colours are
stored as SH DC coefficients: ``dc = (rgb - 0.5) / C0`` inverts
``color_from_dc`` (``spike/forward.py:69-71``).

Cameras follow ``spike/camera.py``: OpenCV world->camera ``R_v[3,3], t_v[3]``, pinhole
``fx, fy, cx, cy``, ``look_at_opencv`` (``spike/camera.py:51-63``) with up = +y.
"""
import math

import numpy as np

C0 = 0.28209479177387814          # spike/sh.py:9


def look_at_opencv(eye, target=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0)):
    """World->camera rotation/translation, float32 (spike/camera.py:51-63)."""
    eye = np.asarray(eye, np.float32)
    target = np.asarray(target, np.float32)
    up = np.asarray(up, np.float32)
    z = target - eye
    z = z / np.linalg.norm(z)
    x = np.cross(up, z)
    x = x / np.linalg.norm(x)
    y = np.cross(z, x)
    R_v = np.stack([x, y, z], 0).astype(np.float32)
    t_v = (-R_v @ eye).astype(np.float32)
    return R_v, t_v


def pinhole(R_v, t_v, H, W, fov_x_deg=50.0):
    """Camera dict with a horizontal field of view; square pixels, centred principal point."""
    fx = 0.5 * W / math.tan(math.radians(fov_x_deg) * 0.5)
    return dict(R_v=np.asarray(R_v, np.float32), t_v=np.asarray(t_v, np.float32),
                fx=float(fx), fy=float(fx), cx=0.5 * W, cy=0.5 * H, H=int(H), W=int(W))


def _unit_quats(rng, G):
    q = rng.standard_normal((G, 4), dtype=np.float32)
    return q / np.linalg.norm(q, axis=1, keepdims=True)


def _sphere_dir(rng):
    v = rng.standard_normal(3)
    return v / np.linalg.norm(v)


def _params(means, log_scales, quats, opacity_raw, rgb, rest):
    G = means.shape[0]
    return dict(
        means3d=np.ascontiguousarray(means, np.float32),
        log_scales=np.ascontiguousarray(log_scales, np.float32),
        quats=np.ascontiguousarray(quats, np.float32),
        opacity_raw=np.ascontiguousarray(opacity_raw, np.float32),
        color_dc=np.ascontiguousarray((rgb - np.float32(0.5)) / np.float32(C0), np.float32),
        color_rest=np.ascontiguousarray(rest if rest is not None else np.zeros((G, 15, 3), np.float32),
                                        np.float32),
        w_b_raw=np.float32(-3.0),
    )


def _clusters(rng, G, n_clusters, sigma, lo=-1.0, hi=1.0):
    centres = rng.uniform(lo, hi, (n_clusters, 3)).astype(np.float32)
    which = rng.integers(0, n_clusters, G)
    return centres[which] + np.float32(sigma) * rng.standard_normal((G, 3), dtype=np.float32)


def config0(seed=0, G=2000, res=128):
    """Config 0: G=2000 uniform in [-1,1]^3, log-scale N(-3.5,0.3), SH deg 0, one 128x128
    camera (fov 50 deg) on the radius-4 sphere looking at the origin; seeded U[0,1] target."""
    rng = np.random.default_rng(seed)
    means = rng.uniform(-1, 1, (G, 3)).astype(np.float32)
    ls = (-3.5 + 0.3 * rng.standard_normal((G, 3))).astype(np.float32)
    q = _unit_quats(rng, G)
    op = rng.standard_normal(G).astype(np.float32)
    rgb = rng.uniform(0, 1, (G, 3)).astype(np.float32)
    eye = 4.0 * _sphere_dir(rng)
    cam = pinhole(*look_at_opencv(eye), res, res)
    target = rng.uniform(0, 1, (res, res, 3)).astype(np.float32)
    return dict(params=_params(means, ls, q, op, rgb, None), sh_degree=0, cams=[cam],
                targets=[target], K=128, R=1)


def config1(seed=1, G=10000, res=800):
    """Config 1: G=10k in 8 isotropic clusters (sigma 0.2), SH deg 3 (rest N(0,0.1), DC colour
    U[0,1]), one 800x800 view; overflowing tiles at K=128."""
    rng = np.random.default_rng(seed)
    means = _clusters(rng, G, 8, 0.2)
    ls = (-3.5 + 0.3 * rng.standard_normal((G, 3))).astype(np.float32)
    q = _unit_quats(rng, G)
    op = rng.standard_normal(G).astype(np.float32)
    rgb = rng.uniform(0, 1, (G, 3)).astype(np.float32)
    rest = (0.1 * rng.standard_normal((G, 15, 3))).astype(np.float32)
    eye = 4.0 * _sphere_dir(rng)
    cam = pinhole(*look_at_opencv(eye), res, res)
    target = rng.uniform(0, 1, (res, res, 3)).astype(np.float32)
    return dict(params=_params(means, ls, q, op, rgb, rest), sh_degree=3, cams=[cam],
                targets=[target], K=128, R=1)


def ring_cameras(rng, n, H, W, radius=4.0, max_elev=0.35):
    """n cameras on a ring of the given radius, azimuth 2*pi*i/n, seeded elevations."""
    cams = []
    for i in range(n):
        az = 2.0 * math.pi * i / n
        el = float(rng.uniform(-max_elev, max_elev))
        eye = radius * np.array([math.cos(el) * math.cos(az), math.sin(el), math.cos(el) * math.sin(az)])
        cams.append(pinhole(*look_at_opencv(eye), H, W))
    return cams


def config2(seed=2, G=100000, H=832, W=1264, n_views=8):
    """Config 2 (the headline train step): G=100k uniform in [-1,1]^3, SH deg 3, 8 cameras on a
    radius-4 ring at seeded elevations, 1264x832 images, K=128, seeded 8-bit target images
    (uniform over 0..255; ``targets_u8`` as drawn, ``targets`` = float32(x) / 255, the [0, 1]
    floats the dataset loaders make of 8-bit frames)."""
    rng = np.random.default_rng(seed)
    means = rng.uniform(-1, 1, (G, 3)).astype(np.float32)
    ls = (-3.5 + 0.3 * rng.standard_normal((G, 3))).astype(np.float32)
    q = _unit_quats(rng, G)
    op = rng.standard_normal(G).astype(np.float32)
    rgb = rng.uniform(0, 1, (G, 3)).astype(np.float32)
    rest = (0.1 * rng.standard_normal((G, 15, 3))).astype(np.float32)
    cams = ring_cameras(rng, n_views, H, W)
    targets_u8 = [rng.integers(0, 256, (H, W, 3), dtype=np.uint8) for _ in range(n_views)]
    targets = [t.astype(np.float32) / np.float32(255.0) for t in targets_u8]
    return dict(params=_params(means, ls, q, op, rgb, rest), sh_degree=3, cams=cams,
                targets=targets, targets_u8=targets_u8, K=128, R=1)


def config3(seed=3, G=1000000, H=1072, W=1920, n_views=1):
    """Config 3: G=1M, 64 tight clusters (sigma 0.05) plus 20% uniform background,
    log-scale N(-4.5,0.5); 1920x1080 cropped to whole tiles (1920x1072), K=256, fp32."""
    rng = np.random.default_rng(seed)
    n_bg = G // 5
    means = np.concatenate([_clusters(rng, G - n_bg, 64, 0.05),
                            rng.uniform(-1, 1, (n_bg, 3)).astype(np.float32)], 0)
    ls = (-4.5 + 0.5 * rng.standard_normal((G, 3))).astype(np.float32)
    q = _unit_quats(rng, G)
    op = rng.standard_normal(G).astype(np.float32)
    rgb = rng.uniform(0, 1, (G, 3)).astype(np.float32)
    cams = [pinhole(*look_at_opencv(4.0 * _sphere_dir(rng)), H, W) for _ in range(n_views)]
    targets = [rng.uniform(0, 1, (H, W, 3)).astype(np.float32) for _ in range(n_views)]
    return dict(params=_params(means, ls, q, op, rgb, None), sh_degree=0, cams=cams,
                targets=targets, K=256, R=1)


def spiral_cameras(rng, n, H, W, radius=6.0):
    """n cameras on a seeded spiral around the origin (radius 6 > 2*sqrt(3), so no gaussian of
    the [-2,2]^3 cube sits behind the near plane)."""
    cams = []
    phase = float(rng.uniform(0, 2 * math.pi))
    for i in range(n):
        s = (i + 0.5) / n
        el = math.asin(1.6 * s - 0.8)
        az = phase + 2.0 * math.pi * 3.0 * s
        eye = radius * np.array([math.cos(el) * math.cos(az), math.sin(el), math.cos(el) * math.sin(az)])
        cams.append(pinhole(*look_at_opencv(eye), H, W))
    return cams


def config4(seed=4, G=3000000, H=832, W=1264, n_views=64):
    """Config 4: batched novel-view render, G=3M uniform in [-2,2]^3, log-scale N(-5,0.4),
    SH deg 3, 64 views at 1264x832 on a seeded spiral (radius 6), K=128, forward only."""
    rng = np.random.default_rng(seed)
    means = rng.uniform(-2, 2, (G, 3)).astype(np.float32)
    ls = (-5.0 + 0.4 * rng.standard_normal((G, 3))).astype(np.float32)
    q = _unit_quats(rng, G)
    op = rng.standard_normal(G).astype(np.float32)
    rgb = rng.uniform(0, 1, (G, 3)).astype(np.float32)
    rest = (0.1 * rng.standard_normal((G, 15, 3))).astype(np.float32)
    cams = spiral_cameras(rng, n_views, H, W)
    return dict(params=_params(means, ls, q, op, rgb, rest), sh_degree=3, cams=cams,
                targets=None, K=128, R=1)


CONFIGS = {0: config0, 1: config1, 2: config2, 3: config3, 4: config4}


def stress_mu2d(seed, G, H, W, n_clusters=16, sigma_px=6.0, frac_off=0.1, frac_drop=0.1,
                n_special=0, quantise=False):
    """2D binning stress input: clustered pixel-space means (many candidates per tile, overflow),
    a fraction pushed off-screen (they clamp into border cells), a fraction with keep=False, and
    optionally special values (nan, +-inf, huge) with keep=True.  ``quantise`` snaps means to a
    1/8-pixel grid so that many candidates share the same quantised distance (ties)."""
    rng = np.random.default_rng(seed)
    centres = np.stack([rng.uniform(0, W, n_clusters), rng.uniform(0, H, n_clusters)], 1)
    which = rng.integers(0, n_clusters, G)
    mu = centres[which] + sigma_px * rng.standard_normal((G, 2))
    off = rng.random(G) < frac_off
    mu[off] = mu[off] * rng.uniform(-3, 4, (int(off.sum()), 1))
    if quantise:
        mu = np.round(mu * 8.0) / 8.0
    mu = mu.astype(np.float32)
    keep = rng.random(G) >= frac_drop
    if n_special:
        specials = np.array([np.nan, np.inf, -np.inf, 1e30, -1e30, 3e19, 9.3e18 * 16, 5e18],
                            np.float32)
        pos = rng.choice(G, size=n_special, replace=False)
        for i, p in enumerate(pos):
            mu[p, i % 2] = specials[i % len(specials)]
            keep[p] = True
    return mu, keep


# ---- the reference's data-free self-consistency scene (spike/synthetic.py:16-48) ---------------
# A known gaussian set rendered from orbit cameras gives ground-truth images that a fresh model
# must recover.  Same names, arguments and draws as the reference; images come from the device
# render.  The default image size is 48 (the reference's 40 rounded up to whole 16-pixel tiles,
# which the binned path needs).

def make_gt_model(seed=1, G=30, extent=0.5, dtype=None, device="cuda"):
    """The known scene: ``GaussianModel(G, extent, seed, gt=True, init_scale=0.08)``."""
    import torch

    from .model import GaussianModel
    if dtype not in (None, torch.float32):
        raise TypeError("the device path keeps gaussians in float32")
    return GaussianModel(G, extent=extent, seed=seed, gt=True, init_scale=0.08, device=device)


def make_orbit_cameras(n=4, radius=2.5, elevation=0.6, res=48, fov=0.7, dtype=None, device=None):
    """n square res x res pinhole cameras (field of view ``fov`` radians, principal point at the
    image centre) at azimuths 2 pi i / n on a ring of the given radius and height, looking at the
    origin.  Cameras stay on the host; the render moves them to the model's device."""
    from .camera import Camera, look_at_opencv as look_at
    f = 0.5 * res / math.tan(0.5 * fov)
    cams = []
    for i in range(n):
        th = 2.0 * math.pi * i / n
        R_v, t_v = look_at((radius * math.cos(th), elevation, radius * math.sin(th)), (0.0, 0.0, 0.0))
        cams.append(Camera(R_v, t_v, f, f, res / 2.0, res / 2.0, res, res))
    return cams


def render_gt_images(gt_model, cameras, arm="A", **kw):
    """One device render per camera, without gradients."""
    import torch

    from .render import render
    with torch.no_grad():
        return [render(gt_model, cam, arm, **kw).detach() for cam in cameras]


def make_scene(arm="A", seed=1, G_gt=30, n_views=4, res=48, device="cuda"):
    """(gt_model, cameras, gt_images) of the self-consistency scene for one arm."""
    gt = make_gt_model(seed=seed, G=G_gt, device=device)
    cams = make_orbit_cameras(n=n_views, res=res)
    return gt, cams, render_gt_images(gt, cams, arm)
