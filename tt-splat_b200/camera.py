"""OpenCV pinhole cameras (the conventions of spike/camera.py) and their device packing.

``Camera`` keeps the reference's fields (world->camera ``R_v[3,3]``, ``t_v[3]`` as torch
tensors, intrinsics, image size) so reference code that builds cameras works unchanged.
``pack_cameras`` lays a list of cameras out as the ``[V, 20]`` float32 device records the
kernels read: R_v (row-major), t_v, fx, fy, cx, cy, centre, pad.
"""
import numpy as np
import torch

CAM_FLOATS = 20


def opengl_c2w_to_opencv_w2c(c2w):
    """OpenGL camera-to-world pose (4x4; camera looks down -z, +y up) -> OpenCV world-to-camera
    (R_v [3,3], t_v [3]; camera looks down +z, +y down).

    A point's OpenCV camera coordinates are its OpenGL camera coordinates with y and z negated,
    so R_v is the transpose of the pose's rotation with its last two rows negated, and
    t_v = -R_v @ (camera position)."""
    c2w = torch.as_tensor(c2w)
    R_v = c2w[:3, :3].transpose(0, 1).clone()
    R_v[1:] = -R_v[1:]
    return R_v, -(R_v @ c2w[:3, 3])


def project_point(p_world, R_v, t_v, fx, fy, cx, cy):
    """Pinhole projection of one world point -> (pixel [2], depth z); z > 0 is in front."""
    x, y, z = R_v @ p_world + t_v
    return torch.stack([fx * x / z + cx, fy * y / z + cy]), z


class Camera:
    """An OpenCV pinhole camera (spike/camera.py:36-48)."""

    __slots__ = ("R_v", "t_v", "fx", "fy", "cx", "cy", "H", "W")

    def __init__(self, R_v, t_v, fx, fy, cx, cy, H, W):
        self.R_v, self.t_v = torch.as_tensor(R_v, dtype=torch.float32), torch.as_tensor(t_v, dtype=torch.float32)
        self.fx, self.fy, self.cx, self.cy = float(fx), float(fy), float(cx), float(cy)
        self.H, self.W = int(H), int(W)

    @property
    def center(self):
        return -self.R_v.transpose(-1, -2) @ self.t_v

    @classmethod
    def from_dict(cls, d):
        return cls(torch.from_numpy(np.asarray(d["R_v"], np.float32)), torch.from_numpy(np.asarray(d["t_v"], np.float32)),
                   d["fx"], d["fy"], d["cx"], d["cy"], d["H"], d["W"])

    def to_dict(self):
        return dict(R_v=self.R_v.detach().cpu().numpy(), t_v=self.t_v.detach().cpu().numpy(), fx=self.fx, fy=self.fy,
                    cx=self.cx, cy=self.cy, H=self.H, W=self.W)

    def record(self):
        """The 20-float device record of this camera."""
        r = np.zeros(CAM_FLOATS, np.float32)
        r[0:9] = self.R_v.detach().cpu().float().reshape(-1).numpy()
        r[9:12] = self.t_v.detach().cpu().float().reshape(-1).numpy()
        r[12:16] = (self.fx, self.fy, self.cx, self.cy)
        r[16:19] = self.center.detach().cpu().float().reshape(-1).numpy()
        return r


def as_camera(c):
    return c if isinstance(c, Camera) else (Camera.from_dict(c) if isinstance(c, dict) else
                                            Camera(c.R_v, c.t_v, c.fx, c.fy, c.cx, c.cy, c.H, c.W))


def pack_cameras(cams, device):
    """[V, 20] float32 device tensor of camera records (all cameras must share H and W)."""
    cams = [as_camera(c) for c in cams]
    H, W = cams[0].H, cams[0].W
    if any(c.H != H or c.W != W for c in cams):
        raise ValueError("all cameras of a batch must share the image size")
    return torch.from_numpy(np.stack([c.record() for c in cams])).to(device)


def look_at_opencv(eye, target, up=(0.0, 1.0, 0.0), dtype=torch.float32, device=None):
    """OpenCV world-to-camera pose (R_v, t_v) of a camera at ``eye`` looking at ``target``: the
    rows of R_v are the camera's right, down and forward axes in world coordinates, with right
    = up x forward (normalised) and down = forward x right."""
    as_vec = lambda v: torch.as_tensor(v, dtype=dtype, device=device)  # noqa: E731
    eye, target, up = as_vec(eye), as_vec(target), as_vec(up)
    forward = target - eye
    forward = forward / forward.norm()
    right = torch.linalg.cross(up, forward)
    right = right / right.norm()
    down = torch.linalg.cross(forward, right)
    R_v = torch.stack([right, down, forward])
    return R_v, -R_v @ eye


def pixel_grid(H, W, dtype=torch.float32, device="cpu"):
    """Pixel centres of an H x W image in row-major order: px [H*W] = column + 0.5,
    py [H*W] = row + 0.5."""
    cols = torch.arange(W, dtype=dtype, device=device) + 0.5
    rows = torch.arange(H, dtype=dtype, device=device) + 0.5
    return cols.repeat(H), rows.repeat_interleave(W)
