"""Tiny seeded on-disk datasets for the loader and .ply tests (no dataset exists in this
environment): a NeRF-synthetic-style split (transforms_train.json + RGBA PNGs) and a COLMAP
sparse model (cameras/images/points3D .bin + RGB PNGs), written in the published formats."""
import json
import math
import os
import struct

import numpy as np
from PIL import Image


def make_blender(root, seed=21, n=3, size=24):
    rng = np.random.default_rng(seed)
    os.makedirs(os.path.join(root, "train"), exist_ok=True)
    frames = []
    for i in range(n):
        rgba = rng.integers(0, 256, (size, size, 4), dtype=np.uint8)
        Image.fromarray(rgba, "RGBA").save(os.path.join(root, "train", f"r_{i}.png"))
        ang = 2 * math.pi * i / n
        c2w = [[math.cos(ang), 0.0, math.sin(ang), 4.0 * math.sin(ang)],
               [0.0, 1.0, 0.0, 0.5 * i],
               [-math.sin(ang), 0.0, math.cos(ang), 4.0 * math.cos(ang)],
               [0.0, 0.0, 0.0, 1.0]]
        frames.append({"file_path": f"./train/r_{i}", "transform_matrix": c2w})
    with open(os.path.join(root, "transforms_train.json"), "w") as f:
        json.dump({"camera_angle_x": 0.6911112070083618, "frames": frames}, f)


def make_colmap(root, seed=22):
    rng = np.random.default_rng(seed)
    sp = os.path.join(root, "sparse", "0")
    os.makedirs(sp, exist_ok=True)
    os.makedirs(os.path.join(root, "images"), exist_ok=True)
    cams = [(1, 1, 32, 24, (30.0, 31.0, 16.0, 12.0)),        # PINHOLE fx fy cx cy
            (2, 0, 32, 24, (28.0, 16.5, 11.5))]              # SIMPLE_PINHOLE f cx cy
    with open(os.path.join(sp, "cameras.bin"), "wb") as f:
        f.write(struct.pack("<Q", len(cams)))
        for cid, model, W, H, p in cams:
            f.write(struct.pack("<iiQQ", cid, model, W, H))
            f.write(struct.pack(f"<{len(p)}d", *p))
    names = ["c.png", "a.png", "b.png"]
    with open(os.path.join(sp, "images.bin"), "wb") as f:
        f.write(struct.pack("<Q", len(names)))
        for k, name in enumerate(names):
            q = rng.standard_normal(4)
            q /= np.linalg.norm(q)
            t = rng.standard_normal(3)
            f.write(struct.pack("<i", k + 1))
            f.write(struct.pack("<4d", *q))
            f.write(struct.pack("<3d", *t))
            f.write(struct.pack("<i", 1 + k % 2))
            f.write(name.encode() + b"\x00")
            npts = int(rng.integers(0, 4))
            f.write(struct.pack("<Q", npts))
            for _ in range(npts):
                f.write(struct.pack("<ddq", *rng.standard_normal(2), int(rng.integers(-1, 50))))
            Image.fromarray(rng.integers(0, 256, (24, 32, 3), dtype=np.uint8), "RGB").save(
                os.path.join(root, "images", name))
    with open(os.path.join(sp, "points3D.bin"), "wb") as f:
        f.write(struct.pack("<Q", 20))
        for i in range(20):
            f.write(struct.pack("<Q", i))
            f.write(struct.pack("<3d", *rng.standard_normal(3)))
            f.write(struct.pack("<3B", *rng.integers(0, 256, 3)))
            f.write(struct.pack("<d", float(rng.random())))
            tl = int(rng.integers(0, 3))
            f.write(struct.pack("<Q", tl))
            for _ in range(tl):
                f.write(struct.pack("<ii", int(rng.integers(1, 4)), int(rng.integers(0, 10))))


def ply_params(seed=23, G=37):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((G, 4)).astype(np.float32)
    q[0] = 0.0                                   # exercises the 1e-12 norm clamp
    return dict(means3d=rng.standard_normal((G, 3)).astype(np.float32),
                log_scales=(rng.standard_normal((G, 3)) - 3).astype(np.float32), quats=q,
                opacity_raw=rng.standard_normal(G).astype(np.float32),
                color_dc=rng.standard_normal((G, 3)).astype(np.float32),
                color_rest=(0.1 * rng.standard_normal((G, 15, 3))).astype(np.float32), w_b_raw=np.float32(-3.0))
