"""Datasets on disk -> (cameras, images) for training and rendering: NeRF-synthetic ("Blender")
splits and COLMAP sparse models, the two formats the reference reads (spike/data.py).

Formats, as published:

* Blender / NeRF-synthetic: ``transforms_<split>.json`` holds ``camera_angle_x`` (horizontal
  field of view, radians) and ``frames``, each with a ``file_path`` (PNG, extension optional) and
  a 4x4 camera-to-world ``transform_matrix`` in the OpenGL convention (camera looks down -z, +y
  up).  Frames are RGBA; the dataset's background is white.
* COLMAP binary sparse model (``sparse/0``), little-endian:
  - ``cameras.bin``: u64 count; per camera i32 id, i32 model, u64 width, u64 height, then the
    model's f64 parameters (count per model below);
  - ``images.bin``: u64 count; per image i32 id, f64 qvec[4] (w, x, y, z), f64 tvec[3], i32
    camera id, NUL-terminated name, u64 number of 2-D points, then (f64 x, f64 y, i64 point id)
    per point.  (qvec, tvec) is the world-to-camera pose in the OpenCV convention, which is
    the convention of ``camera.Camera``;
  - ``points3D.bin``: u64 count; per point u64 id, f64 xyz[3], u8 rgb[3], f64 error, u64 track
    length, then (i32 image id, i32 point2D index) per track element.

Images come back as float32 tensors in [0, 1] on ``device`` ([H,W,3], or straight RGBA [H,W,4]
with ``keep_alpha``), bit-identical to the reference loader's output on the same files (same
PIL resampling, /255 in float32, "over white" compositing rgb*a + (1-a)).  This is host IO;
the training step consumes the returned tensors.
"""
import json
import math
import os
import struct

import numpy as np
import torch
from PIL import Image

from .camera import Camera, opengl_c2w_to_opencv_w2c

# COLMAP camera models: id -> (name, number of parameters, single focal length?)
COLMAP_MODELS = {
    0: ("SIMPLE_PINHOLE", 3, True), 1: ("PINHOLE", 4, False), 2: ("SIMPLE_RADIAL", 4, True),
    3: ("RADIAL", 5, True), 4: ("OPENCV", 8, False), 5: ("OPENCV_FISHEYE", 8, False),
    6: ("FULL_OPENCV", 12, False), 7: ("FOV", 5, False), 8: ("SIMPLE_RADIAL_FISHEYE", 4, True),
    9: ("RADIAL_FISHEYE", 5, True), 10: ("THIN_PRISM_FISHEYE", 12, False),
}


# ---- Blender / NeRF-synthetic -----------------------------------------------------------------
def intrinsics_from_fov(camera_angle_x, W, H):
    """Square-pixel pinhole (fx, fy, cx, cy) whose horizontal field of view is camera_angle_x,
    principal point at the image centre."""
    focal = 0.5 * W / math.tan(0.5 * camera_angle_x)
    return focal, focal, W / 2.0, H / 2.0


def composite_over_white(rgba):
    """Straight-alpha RGBA [...,4] -> RGB [...,3] over a white background."""
    alpha = rgba[..., 3:4]
    return rgba[..., :3] * alpha + (1.0 - alpha)


def select_indices(n_frames, indices=None, stride=None, n=None):
    """Frame selection shared by the loaders: ``indices`` as given, else every ``stride``-th
    frame (all when None), the first ``n`` of those when ``n`` is given."""
    if indices is not None:
        return list(indices)
    picked = list(range(n_frames))[::stride or 1]
    return picked if n is None else picked[:n]


def _rgba_frame(path, res, dtype):
    """A PNG as float RGBA in [0,1], resized (bilinear) to res x res when res is given."""
    with Image.open(path) as im:
        im = im.convert("RGBA")
        if res is not None and im.size != (res, res):
            im = im.resize((res, res), Image.BILINEAR)
        pixels = np.asarray(im, dtype=np.float32)
    return torch.from_numpy(pixels).to(dtype) / 255.0


def load_blender(root, split="train", res=200, indices=None, stride=None, n=None, device="cpu",
                 dtype=torch.float32, keep_alpha=False):
    """A NeRF-synthetic split -> (cameras, images).  Poses are converted from OpenGL
    camera-to-world to OpenCV world-to-camera; frames are resized to ``res`` (None keeps the file
    size) and composited over white unless ``keep_alpha``."""
    with open(os.path.join(root, f"transforms_{split}.json")) as f:
        meta = json.load(f)
    fov = meta["camera_angle_x"]
    frames = meta["frames"]
    cameras, images = [], []
    for i in select_indices(len(frames), indices, stride, n):
        frame = frames[i]
        rel = frame["file_path"]
        if not rel.endswith(".png"):
            rel += ".png"
        rgba = _rgba_frame(os.path.normpath(os.path.join(root, rel)), res, dtype)
        img = (rgba if keep_alpha else composite_over_white(rgba)).to(device)
        pose = torch.tensor(frame["transform_matrix"], dtype=dtype, device=device)
        R_v, t_v = opengl_c2w_to_opencv_w2c(pose)
        height, width = img.shape[0], img.shape[1]
        cameras.append(Camera(R_v, t_v, *intrinsics_from_fov(fov, width, height), height, width))
        images.append(img)
    return cameras, images


# ---- COLMAP binary sparse model -------------------------------------------------------------------
class _Cursor:
    """Sequential little-endian reader over a whole file's bytes."""

    def __init__(self, path):
        with open(path, "rb") as f:
            self.buf = f.read()
        self.pos = 0

    def take(self, fmt):
        vals = struct.unpack_from("<" + fmt, self.buf, self.pos)
        self.pos += struct.calcsize("<" + fmt)
        return vals

    def skip(self, nbytes):
        self.pos += nbytes

    def cstring(self):
        end = self.buf.index(b"\0", self.pos)
        s = self.buf[self.pos:end].decode()
        self.pos = end + 1
        return s


def read_colmap_cameras(path):
    """cameras.bin -> {camera id: (fx, fy, cx, cy, width, height)}.  Models with one focal
    length (f, cx, cy, ...) give fx = fy = f; the others start with fx, fy, cx, cy."""
    cur = _Cursor(path)
    (count,) = cur.take("Q")
    cams = {}
    for _ in range(count):
        cid, model, width, height = cur.take("iiQQ")
        if model not in COLMAP_MODELS:
            raise ValueError(f"{path}: unknown COLMAP camera model {model}")
        _, n_params, single = COLMAP_MODELS[model]
        p = cur.take(f"{n_params}d")
        fx, fy, cx, cy = (p[0], p[0], p[1], p[2]) if single else p[:4]
        cams[cid] = (fx, fy, cx, cy, width, height)
    return cams


def read_colmap_images(path):
    """images.bin -> [(qvec, tvec, camera id, name)] in file order (2-D points skipped)."""
    cur = _Cursor(path)
    (count,) = cur.take("Q")
    out = []
    for _ in range(count):
        cur.skip(4)                                    # image id
        vals = cur.take("4d3di")
        name = cur.cstring()
        (n_points,) = cur.take("Q")
        cur.skip(24 * n_points)
        out.append((np.array(vals[0:4]), np.array(vals[4:7]), vals[7], name))
    return out


def qvec_to_rotmat(qvec):
    """Rotation matrix (float64) of a COLMAP unit quaternion (w, x, y, z): the standard
    quaternion-to-matrix formula."""
    w, x, y, z = (float(c) for c in qvec)
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]], np.float64)


def load_colmap(root, downscale=1, n=None, stride=None, device="cpu", dtype=torch.float32):
    """A COLMAP scene (root/sparse/0 + root/images) -> (cameras, images [H,W,3] in [0,1]), views in
    image-name order; an integer ``downscale`` divides the resolution (bilinear) and the
    intrinsics."""
    sparse = os.path.join(root, "sparse", "0")
    intr = read_colmap_cameras(os.path.join(sparse, "cameras.bin"))
    views = sorted(read_colmap_images(os.path.join(sparse, "images.bin")), key=lambda v: v[3])
    cameras, images = [], []
    for i in select_indices(len(views), None, stride, n):
        qvec, tvec, cid, name = views[i]
        fx, fy, cx, cy, width, height = intr[cid]
        with Image.open(os.path.join(root, "images", name)) as im:
            im = im.convert("RGB")
            if downscale > 1:
                width, height = width // downscale, height // downscale
                im = im.resize((width, height), Image.BILINEAR)
                scale = 1.0 / downscale
                fx, fy, cx, cy = fx * scale, fy * scale, cx * scale, cy * scale
            pixels = np.asarray(im, dtype=np.float32) / 255.0
        img = torch.from_numpy(pixels).to(dtype).to(device)
        R_v = torch.from_numpy(qvec_to_rotmat(qvec)).to(dtype).to(device)
        t_v = torch.from_numpy(np.asarray(tvec, np.float64)).to(dtype).to(device)
        cameras.append(Camera(R_v, t_v, float(fx), float(fy), float(cx), float(cy), int(height), int(width)))
        images.append(img)
    return cameras, images


def load_colmap_points(root, max_pts=None):
    """points3D.bin -> (xyz [N,3] float32, rgb [N,3] float32 in [0,1]) for gaussian
    initialisation; with ``max_pts`` a seeded subset (numpy default_rng(0), no repeats, the
    reference's choice) of that many points."""
    cur = _Cursor(os.path.join(root, "sparse", "0", "points3D.bin"))
    (count,) = cur.take("Q")
    xyz = np.empty((count, 3), np.float64)
    rgb = np.empty((count, 3), np.uint8)
    for i in range(count):
        vals = cur.take("Q3d3Bd")
        xyz[i], rgb[i] = vals[1:4], vals[4:7]
        (track,) = cur.take("Q")
        cur.skip(8 * track)
    xyz = xyz.astype(np.float32)
    rgb = rgb.astype(np.float32) / 255.0
    if max_pts and count > max_pts:
        keep = np.random.default_rng(0).choice(count, max_pts, replace=False)
        xyz, rgb = xyz[keep], rgb[keep]
    return xyz, rgb
