"""Dataset loaders and .ply IO against the reference's own outputs (tests/golden/io.npz, made by
make_golden_io.py from spike/data.py and spike/plyio.py on the seeded datasets of
io_datasets.py).  Host code: runs on CPU."""
import os

import numpy as np
import pytest
import torch

from conftest import golden
import io_datasets


@pytest.fixture(scope="module")
def z():
    return golden("io.npz")


def _check(z, tag, cams, imgs):
    assert np.array_equal(np.stack([c.R_v.numpy() for c in cams]), z[f"{tag}__R"])
    assert np.array_equal(np.stack([c.t_v.numpy() for c in cams]), z[f"{tag}__t"])
    assert np.array_equal(np.array([[c.fx, c.fy, c.cx, c.cy, c.H, c.W] for c in cams], np.float64), z[f"{tag}__k"])
    assert np.array_equal(np.stack([i.numpy() for i in imgs]), z[f"{tag}__img"])


def test_blender_loader_matches_reference(z, tmp_path, pkg):
    from tt_splat_b200 import data
    root = str(tmp_path / "blender")
    io_datasets.make_blender(root)
    for tag, kw in (("b_full", dict(res=None)), ("b_res16", dict(res=16)), ("b_alpha", dict(res=None, keep_alpha=True)),
                    ("b_stride", dict(res=None, stride=2))):
        cams, imgs = data.load_blender(root, "train", **kw)
        _check(z, tag, cams, imgs)


def test_colmap_loader_matches_reference(z, tmp_path, pkg):
    from tt_splat_b200 import data
    root = str(tmp_path / "colmap")
    io_datasets.make_colmap(root)
    for tag, kw in (("c_full", dict()), ("c_down2", dict(downscale=2))):
        cams, imgs = data.load_colmap(root, **kw)
        _check(z, tag, cams, imgs)
    xyz, rgb = data.load_colmap_points(root)
    assert np.array_equal(xyz, z["pts__xyz"]) and np.array_equal(rgb, z["pts__rgb"])
    xyz, rgb = data.load_colmap_points(root, max_pts=7)
    assert np.array_equal(xyz, z["pts7__xyz"]) and np.array_equal(rgb, z["pts7__rgb"])


def test_save_ply_is_byte_identical_to_reference(z, tmp_path, pkg):
    from tt_splat_b200 import plyio
    from tt_splat_b200.model import GaussianModel
    p = io_datasets.ply_params()
    m = GaussianModel.from_arrays(p, device="cpu")
    path = str(tmp_path / "m.ply")
    assert plyio.save_ply(path, m) == p["means3d"].shape[0]
    assert open(path, "rb").read() == z["ply_bytes"].tobytes()


def test_ply_round_trip(tmp_path, pkg):
    from tt_splat_b200 import plyio
    from tt_splat_b200.model import GaussianModel
    p = io_datasets.ply_params()
    m = GaussianModel.from_arrays(p, device="cpu")
    for sh_rest in (False, True):
        path = str(tmp_path / f"m{int(sh_rest)}.ply")
        plyio.save_ply(path, m, sh_rest=sh_rest)
        back = plyio.load_ply(path, device="cpu").to_arrays()
        for k in ("means3d", "log_scales", "opacity_raw", "color_dc"):
            assert np.array_equal(back[k], p[k]), k
        q = torch.from_numpy(p["quats"])
        qn = (q / q.norm(dim=-1, keepdim=True).clamp(min=1e-12)).numpy()
        assert np.array_equal(back["quats"], qn)
        rest = back["color_rest"]
        assert np.array_equal(rest, p["color_rest"] if sh_rest else np.zeros_like(p["color_rest"]))


def test_ply_reader_rejects_other_formats(tmp_path, pkg):
    from tt_splat_b200 import plyio
    bad = tmp_path / "a.ply"
    bad.write_bytes(b"ply\nformat ascii 1.0\nelement vertex 1\nproperty float x\nend_header\n1.0\n")
    with pytest.raises(ValueError):
        plyio.load_ply(str(bad), device="cpu")
