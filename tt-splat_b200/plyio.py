"""The trained model on disk: standard binary 3DGS .ply (mirrors spike/plyio.py:1-42).

``save_ply(path, model)`` writes the reference's layout byte for byte: a binary_little_endian
header with one ``element vertex`` of 17 float properties — x, y, z, nx, ny, nz (zero), f_dc_0..2
(the SH DC colour), opacity (the logit), scale_0..2 (log scales), rot_0..3 (the quaternion
normalised with the norm clamped at 1e-12) — DC only, like the reference.  ``sh_rest=True``
appends the standard f_rest_0..44 properties (channel-major, the 3DGS convention) so an SH model
round-trips; readers that expect the reference's 17 fields must then be given the extended
header.  ``load_ply(path)`` reads either layout (the reader of
tools/gsplat_sweep_views.py:32-53 handles the 17-field one) back into a ``GaussianModel``.

The parameters are read from the device once; the file IO is host work.
"""
import re

import numpy as np
import torch

from .model import GaussianModel, flat_of, view

_FIELDS = (["x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2", "opacity"]
           + [f"scale_{i}" for i in range(3)] + [f"rot_{i}" for i in range(4)])
_REST = [f"f_rest_{i}" for i in range(45)]


def _params_of(model):
    """(means3d, color_dc, opacity_raw, log_scales, quats, color_rest) as CPU float32 tensors from a
    tt_splat_b200 GaussianModel or any object with the reference's parameter attributes."""
    if isinstance(model, GaussianModel):
        flat = flat_of(model).detach().float().cpu()
        G = model.G
        get = lambda n: view(flat, G, n)  # noqa: E731
    else:
        get = lambda n: getattr(model, n).detach().float().cpu()  # noqa: E731
    rest = get("color_rest") if isinstance(model, GaussianModel) or hasattr(model, "color_rest") else None
    return get("means3d"), get("color_dc"), get("opacity_raw"), get("log_scales"), get("quats"), rest


@torch.no_grad()
def save_ply(path, model, sh_rest=False):
    """Write ``model`` to ``path`` as a binary_little_endian 3DGS .ply; returns the gaussian count
    (spike/plyio.py:21-42)."""
    xyz, f_dc, op, ls, q, rest = _params_of(model)
    n = xyz.shape[0]
    q = q / q.norm(dim=-1, keepdim=True).clamp(min=1e-12)          # normalised quaternion
    cols = [xyz.numpy(), np.zeros((n, 3), np.float32), f_dc.numpy(), op.reshape(n, 1).numpy(), ls.numpy(),
            q.numpy()]
    names = list(_FIELDS)
    if sh_rest:
        r = (rest if rest is not None else torch.zeros(n, 15, 3)).reshape(n, 15, 3)
        cols.append(r.permute(0, 2, 1).reshape(n, 45).numpy())      # f_rest channel-major
        names += _REST
    data = np.concatenate(cols, axis=1).astype("<f4")
    header = ("ply\nformat binary_little_endian 1.0\n"
              f"element vertex {n}\n"
              + "".join(f"property float {f}\n" for f in names)
              + "end_header\n")
    with open(path, "wb") as fh:
        fh.write(header.encode("ascii"))
        fh.write(data.tobytes())
    return n


def read_ply_arrays(path):
    """Parse a binary_little_endian float .ply with a single vertex element -> {property: array}."""
    with open(path, "rb") as fh:
        if fh.readline().strip() != b"ply":
            raise ValueError(f"{path}: not a .ply file")
        n, props, fmt = None, [], None
        while True:
            line = fh.readline()
            if not line:
                raise ValueError(f"{path}: truncated header")
            line = line.strip()
            if line.startswith(b"format"):
                fmt = line.split()[1]
            elif line.startswith(b"element vertex"):
                n = int(line.split()[-1])
            elif line.startswith(b"property"):
                parts = line.split()
                if parts[1] != b"float":
                    raise ValueError(f"{path}: only float properties are supported ({line.decode()})")
                props.append(parts[2].decode())
            elif line == b"end_header":
                break
        if fmt != b"binary_little_endian" or n is None:
            raise ValueError(f"{path}: expected a binary_little_endian vertex element")
        raw = np.frombuffer(fh.read(n * len(props) * 4), dtype="<f4")
        if raw.size != n * len(props):
            raise ValueError(f"{path}: {raw.size} values for {n} x {len(props)}")
    raw = raw.reshape(n, len(props))
    return {p: raw[:, i] for i, p in enumerate(props)}


def load_ply(path, device="cuda", w_b_raw=-3.0):
    """Read a 3DGS .ply (the layout ``save_ply`` writes, with or without f_rest) into a
    ``GaussianModel`` on ``device``; absent SH rest coefficients are zero, w_b_raw is the model
    default (spike/model.py:47)."""
    a = read_ply_arrays(path)
    stack = lambda names: np.stack([a[k] for k in names], 1).astype(np.float32)  # noqa: E731
    n = a["x"].shape[0]
    rest_names = sorted((k for k in a if re.fullmatch(r"f_rest_\d+", k)), key=lambda k: int(k.split("_")[-1]))
    rest = np.zeros((n, 15, 3), np.float32)
    if rest_names:
        if len(rest_names) != 45:
            raise ValueError(f"{path}: {len(rest_names)} f_rest properties (expected 45 for SH degree 3)")
        rest = stack(rest_names).reshape(n, 3, 15).transpose(0, 2, 1).copy()
    params = dict(means3d=stack(["x", "y", "z"]), log_scales=stack([f"scale_{i}" for i in range(3)]),
                  quats=stack([f"rot_{i}" for i in range(4)]), opacity_raw=a["opacity"].astype(np.float32).copy(),
                  color_dc=stack(["f_dc_0", "f_dc_1", "f_dc_2"]), color_rest=rest, w_b_raw=np.float32(w_b_raw))
    return GaussianModel.from_arrays(params, device=device)
