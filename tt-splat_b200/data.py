"""Datasets on disk -> (cameras, images) for training and rendering (mirrors spike/data.py:1-171).

* ``load_blender``: NeRF-synthetic splits — transforms_{split}.json + RGBA PNG frames; each
  Blender/OpenGL camera-to-world pose becomes an OpenCV world-to-camera pose
  (``camera.opengl_c2w_to_opencv_w2c``), frames are resized to ``res`` (bilinear) and composited
  over white, intrinsics follow the horizontal field of view (spike/data.py:19-82).
* ``load_colmap`` / ``load_colmap_points``: COLMAP sparse models (sparse/0/{cameras,images,
  points3D}.bin) and their images; COLMAP's world-to-camera convention is the cameras' own
  (spike/data.py:85-171).

Images come back as float32 tensors in [0, 1] on ``device`` ([H,W,3], or [H,W,4] straight RGBA
with ``keep_alpha``).  This is host IO (PIL + struct), as in the reference; the training step
consumes the returned tensors.
"""
import json
import math
import os
import struct

import numpy as np
import torch
from PIL import Image

from .camera import Camera, opengl_c2w_to_opencv_w2c


def intrinsics_from_fov(camera_angle_x, W, H):
    """Pinhole intrinsics from the horizontal field of view (square pixels), spike/data.py:19-22."""
    fx = 0.5 * W / math.tan(0.5 * camera_angle_x)
    return fx, fx, W / 2.0, H / 2.0


def composite_over_white(rgba):
    """rgba [...,4] in [0,1] -> rgb [...,3] over a white background (spike/data.py:25-28)."""
    rgb, a = rgba[..., :3], rgba[..., 3:4]
    return rgb * a + (1.0 - a)


def _load_rgba(path, res, dtype, keep_alpha):
    img = Image.open(path).convert("RGBA")
    if res is not None and (img.width != res or img.height != res):
        img = img.resize((res, res), Image.BILINEAR)
    arr = torch.from_numpy(np.asarray(img, dtype=np.float32)).to(dtype) / 255.0
    return arr if keep_alpha else composite_over_white(arr)


def select_indices(n_frames, indices=None, stride=None, n=None):
    """Deterministic frame selection: explicit indices, or every ``stride``-th, capped at ``n``."""
    if indices is not None:
        return list(indices)
    idx = list(range(0, n_frames, stride)) if stride else list(range(n_frames))
    return idx[:n] if n is not None else idx


def load_blender(root, split="train", res=200, indices=None, stride=None, n=None, device="cpu",
                 dtype=torch.float32, keep_alpha=False):
    """A NeRF-synthetic split -> (cameras, images) (spike/data.py:48-82)."""
    with open(os.path.join(root, f"transforms_{split}.json")) as f:
        meta = json.load(f)
    frames = meta["frames"]
    cameras, images = [], []
    for i in select_indices(len(frames), indices, stride, n):
        fr = frames[i]
        c2w = torch.tensor(fr["transform_matrix"], dtype=dtype, device=device)
        R_v, t_v = opengl_c2w_to_opencv_w2c(c2w)
        fp = fr["file_path"]
        png = os.path.normpath(os.path.join(root, fp if fp.endswith(".png") else fp + ".png"))
        img = _load_rgba(png, res, dtype, keep_alpha).to(device)
        H, W = img.shape[0], img.shape[1]
        fx, fy, cx, cy = intrinsics_from_fov(meta["camera_angle_x"], W, H)
        cameras.append(Camera(R_v, t_v, fx, fy, cx, cy, H, W))
        images.append(img)
    return cameras, images


# ---- COLMAP sparse models (binary) -------------------------------------------------------------
# cameras.bin: u64 count, then per camera i32 id, i32 model, u64 width, u64 height, f64 params[];
# images.bin: u64 count, then per image i32 id, f64 qvec[4] (w,x,y,z), f64 tvec[3], i32 camera id,
# NUL-terminated name, u64 n_points2D, (f64 x, f64 y, i64 point3D id) per point;
# points3D.bin: u64 count, then per point u64 id, f64 xyz[3], u8 rgb[3], f64 error, u64 track
# length, (i32 image id, i32 point2D index) per track element.
_N_PARAMS = {0: 3, 1: 4, 2: 4, 3: 5, 4: 8}


def qvec_to_rotmat(q):
    """COLMAP quaternion (w, x, y, z) -> rotation matrix (float64)."""
    w, x, y, z = q
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]], dtype=np.float64)


def read_colmap_cameras(path):
    """camera id -> (fx, fy, cx, cy, W, H); SIMPLE_PINHOLE/SIMPLE_RADIAL carry one focal length."""
    cams = {}
    with open(path, "rb") as f:
        (count,) = struct.unpack("<Q", f.read(8))
        for _ in range(count):
            cid, model = struct.unpack("<ii", f.read(8))
            W, H = struct.unpack("<QQ", f.read(16))
            k = _N_PARAMS.get(model, 4)
            p = struct.unpack(f"<{k}d", f.read(8 * k))
            if model in (0, 2):
                fx = fy = p[0]
                cx, cy = p[1], p[2]
            else:
                fx, fy, cx, cy = p[0], p[1], p[2], p[3]
            cams[cid] = (fx, fy, cx, cy, W, H)
    return cams


def read_colmap_images(path):
    """[(qvec, tvec, camera id, name)] in file order."""
    out = []
    with open(path, "rb") as f:
        (count,) = struct.unpack("<Q", f.read(8))
        for _ in range(count):
            f.read(4)
            q = struct.unpack("<4d", f.read(32))
            t = struct.unpack("<3d", f.read(24))
            (cid,) = struct.unpack("<i", f.read(4))
            name = bytearray()
            while True:
                c = f.read(1)
                if c in (b"\x00", b""):
                    break
                name += c
            (npts,) = struct.unpack("<Q", f.read(8))
            f.read(24 * npts)
            out.append((np.array(q), np.array(t), cid, name.decode()))
    return out


def load_colmap(root, downscale=1, n=None, stride=None, device="cpu", dtype=torch.float32):
    """A COLMAP scene (root/sparse/0 + root/images) -> (cameras, images [H,W,3] in [0,1]), views
    sorted by image name; ``downscale`` divides the resolution and intrinsics by an integer."""
    sp = os.path.join(root, "sparse", "0")
    cams = read_colmap_cameras(os.path.join(sp, "cameras.bin"))
    meta = sorted(read_colmap_images(os.path.join(sp, "images.bin")), key=lambda r: r[3])
    cameras, images = [], []
    for i in select_indices(len(meta), None, stride, n):
        q, t, cid, name = meta[i]
        fx, fy, cx, cy, W, H = cams[cid]
        im = Image.open(os.path.join(root, "images", name)).convert("RGB")
        if downscale > 1:
            W, H = W // downscale, H // downscale
            im = im.resize((W, H), Image.BILINEAR)
            s = 1.0 / downscale
            fx, fy, cx, cy = fx * s, fy * s, cx * s, cy * s
        arr = torch.from_numpy(np.asarray(im, dtype=np.float32) / 255.0).to(dtype).to(device)
        R_v = torch.from_numpy(qvec_to_rotmat(q)).to(dtype).to(device)
        t_v = torch.from_numpy(t).to(dtype).to(device)
        cameras.append(Camera(R_v, t_v, float(fx), float(fy), float(cx), float(cy), int(H), int(W)))
        images.append(arr)
    return cameras, images


def load_colmap_points(root, max_pts=None):
    """sparse/0/points3D.bin -> (xyz [N,3] float32, rgb [N,3] in [0,1]); ``max_pts`` keeps a seeded
    random subset (numpy default_rng(0), as the reference) for gaussian initialisation."""
    xyz, rgb = [], []
    with open(os.path.join(root, "sparse", "0", "points3D.bin"), "rb") as f:
        (count,) = struct.unpack("<Q", f.read(8))
        for _ in range(count):
            f.read(8)
            xyz.append(struct.unpack("<3d", f.read(24)))
            rgb.append(struct.unpack("<3B", f.read(3)))
            f.read(8)
            (tlen,) = struct.unpack("<Q", f.read(8))
            f.read(8 * tlen)
    xyz = np.array(xyz, dtype=np.float32).reshape(-1, 3)
    rgb = np.array(rgb, dtype=np.float32).reshape(-1, 3) / 255.0
    if max_pts and len(xyz) > max_pts:
        sel = np.random.default_rng(0).choice(len(xyz), max_pts, replace=False)
        xyz, rgb = xyz[sel], rgb[sel]
    return xyz, rgb
