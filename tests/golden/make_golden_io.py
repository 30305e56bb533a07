"""Golden outputs of the reference's dataset loaders and .ply writer (spike/data.py,
spike/plyio.py) on the seeded datasets of io_datasets.py.

    python tests/golden/make_golden_io.py --reference <path to the kinginu/tt-splat checkout>
"""
import argparse
import os
import sys
import tempfile
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import io_datasets  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from spike import data, plyio
    out = {}
    with tempfile.TemporaryDirectory() as d:
        bl = os.path.join(d, "blender")
        io_datasets.make_blender(bl)
        for tag, kw in (("b_full", dict(res=None)), ("b_res16", dict(res=16)), ("b_alpha", dict(res=None, keep_alpha=True)),
                        ("b_stride", dict(res=None, stride=2))):
            cams, imgs = data.load_blender(bl, "train", **kw)
            out[f"{tag}__R"] = np.stack([c.R_v.numpy() for c in cams])
            out[f"{tag}__t"] = np.stack([c.t_v.numpy() for c in cams])
            out[f"{tag}__k"] = np.array([[c.fx, c.fy, c.cx, c.cy, c.H, c.W] for c in cams], np.float64)
            out[f"{tag}__img"] = np.stack([i.numpy() for i in imgs])
        cm = os.path.join(d, "colmap")
        io_datasets.make_colmap(cm)
        for tag, kw in (("c_full", dict()), ("c_down2", dict(downscale=2))):
            cams, imgs = data.load_colmap(cm, **kw)
            out[f"{tag}__R"] = np.stack([c.R_v.numpy() for c in cams])
            out[f"{tag}__t"] = np.stack([c.t_v.numpy() for c in cams])
            out[f"{tag}__k"] = np.array([[c.fx, c.fy, c.cx, c.cy, c.H, c.W] for c in cams], np.float64)
            out[f"{tag}__img"] = np.stack([i.numpy() for i in imgs])
        xyz, rgb = data.load_colmap_points(cm)
        out["pts__xyz"], out["pts__rgb"] = xyz, rgb
        xyz, rgb = data.load_colmap_points(cm, max_pts=7)
        out["pts7__xyz"], out["pts7__rgb"] = xyz, rgb
        p = io_datasets.ply_params()
        m = types.SimpleNamespace(**{k: torch.from_numpy(v) for k, v in p.items() if k != "w_b_raw"})
        path = os.path.join(d, "m.ply")
        plyio.save_ply(path, m)
        out["ply_bytes"] = np.frombuffer(open(path, "rb").read(), np.uint8)
    np.savez_compressed(os.path.join(HERE, "io.npz"), **out)
    print("wrote", os.path.join(HERE, "io.npz"), len(out), "arrays")


if __name__ == "__main__":
    main()
