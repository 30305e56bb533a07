"""Golden outputs of the reference's model initialisation and synthetic-scene cameras:
``GaussianModel(G, extent, seed, gt, init_scale)`` draws (spike/model.py:16-51),
``GaussianModel.init_from_points`` on seeded point clouds (spike/model.py:55-79) and
``synthetic.make_orbit_cameras`` (spike/synthetic.py:20-30).

    python tests/golden/make_golden_scene.py --reference <path to the kinginu/tt-splat checkout>

The reference is imported unmodified; ``ttnn`` and ``pytorch_msssim`` are stubbed in
``sys.modules`` before import (neither is used by the functions called here).
"""
import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

MODEL_CASES = {            # name: (G, extent, seed, gt, init_scale)
    "m_g40": (40, 0.6, 5, True, 0.05),
    "m_fresh150": (150, 0.7, 2, False, 0.05),
    "m_gt30": (30, 0.5, 1, True, 0.08),
    "m_default4": (4, 1.3, 3, False, 0.05),
}
ORBIT_CASES = {            # name: make_orbit_cameras keyword arguments
    "o_default48": dict(n=4, res=48),
    "o_custom": dict(n=3, radius=3.0, elevation=0.2, res=32, fov=0.9),
}
POINT_CASES = {            # name: (points P, gaussians G, cloud seed, init seed)
    "p_subset": (500, 200, 11, 7),
    "p_pad": (50, 120, 12, 3),
}


def point_cloud(P, seed):
    rng = np.random.default_rng(seed)
    xyz = rng.normal(0.0, 0.8, (P, 3)).astype(np.float32)
    rgb = (rng.integers(0, 256, (P, 3)).astype(np.float32) / 255.0).astype(np.float32)
    return xyz, rgb


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.modules.setdefault("ttnn", types.ModuleType("ttnn"))
    sys.modules.setdefault("pytorch_msssim", types.ModuleType("pytorch_msssim"))
    sys.path.insert(0, args.reference)
    from spike import synthetic
    from spike.model import GaussianModel
    out = {}
    for name, (G, extent, seed, gt, init_scale) in MODEL_CASES.items():
        m = GaussianModel(G, extent=extent, seed=seed, gt=gt, init_scale=init_scale)
        for f in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc"):
            out[f"{name}__{f}"] = getattr(m, f).detach().numpy()
    for name, kw in ORBIT_CASES.items():
        cams = synthetic.make_orbit_cameras(**kw)
        out[f"{name}__R"] = np.stack([c.R_v.numpy() for c in cams])
        out[f"{name}__t"] = np.stack([c.t_v.numpy() for c in cams])
        out[f"{name}__k"] = np.array([[c.fx, c.fy, c.cx, c.cy, c.H, c.W] for c in cams], np.float64)
    for name, (P, G, cseed, iseed) in POINT_CASES.items():
        xyz, rgb = point_cloud(P, cseed)
        m = GaussianModel(G, seed=0).init_from_points(torch.from_numpy(xyz), torch.from_numpy(rgb), seed=iseed)
        for f in ("means3d", "log_scales", "color_dc"):
            out[f"{name}__{f}"] = m.__getattr__(f).detach().numpy()
    np.savez_compressed(os.path.join(HERE, "scene.npz"), **out)
    print(f"wrote {len(out)} arrays to scene.npz")


if __name__ == "__main__":
    main()
