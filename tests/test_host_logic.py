"""Host-side logic that needs no GPU: cached binning tables, device guards, view partitions."""
import math

import pytest
import torch


def test_cached_table_format_and_validation(pkg):
    """The reference's (idx, valid) pair -> int32 ids with -1 where invalid (valid slots first);
    holes, out-of-range ids and wrong shapes are rejected before any launch."""
    from tt_splat_b200.binned import _cached_table
    T, K, G = 3, 4, 10
    idx = torch.tensor([[5, 2, 0, 0], [9, 0, 0, 0], [0, 0, 0, 0]])
    valid = torch.tensor([[True, True, False, False], [True, False, False, False], [False] * 4])
    t = _cached_table((idx, valid), G, T, K, "cpu")
    assert t.dtype == torch.int32 and tuple(t.shape) == (1, T, K)
    assert t[0].tolist() == [[5, 2, -1, -1], [9, -1, -1, -1], [-1, -1, -1, -1]]
    hole = valid.clone()
    hole[0, 0] = False
    with pytest.raises(ValueError):
        _cached_table((idx, hole), G, T, K, "cpu")
    with pytest.raises(ValueError):
        _cached_table((idx, valid), 5, T, K, "cpu")            # id 9 >= G
    with pytest.raises(ValueError):
        _cached_table((idx[:, :3], valid[:, :3]), G, T, K, "cpu")


def test_device_guard_is_a_no_op_for_cpu_tensors(pkg):
    from tt_splat_b200._lib import on_device
    with on_device(torch.zeros(1)):
        pass
    with on_device(None):
        pass


def test_ops_reject_cpu_tensors(pkg):
    """No CPU fallback: a CPU tensor reaching an op raises before the library is called."""
    from tt_splat_b200 import ops
    with pytest.raises(RuntimeError):
        ops._dev(torch.zeros(4))


def test_cpu_baseline_step_matches_serial_oracle(pkg):
    """The benchmark's CPU baseline (views over spawned workers, gradients summed in view order)
    computes the same step as the serial oracle: same loss, same Adam update."""
    import numpy as np
    from oracle import loss as oloss
    from oracle import pipeline as opipe
    from oracle.step import LR, CpuStep
    sc = pkg.synthetic.config2(G=3000, H=64, W=96, n_views=3)
    with CpuStep(sc, workers=2) as cs:
        loss, q = cs.step()
    p = sc["params"]
    g, total = None, 0.0
    for v in range(3):
        fw = opipe.render_view(p, 3, sc["cams"][v], K=128)
        lv, _, _, gimg = oloss.loss_and_grad(fw["img"], sc["targets"][v], 0.2)
        gv = opipe.backward_view(fw, (gimg / 3).astype(np.float32), p, 3)
        g = gv if g is None else {k: g[k] + gv[k] for k in g}
        total += lv
    assert abs(loss - total / 3) < 1e-12
    ref = opipe.copy_params(p)
    opipe.adam_step(ref, g, {}, 1, LR, 3)
    # SGLD noise and relocation move means and may overwrite relocated rows; the colours of
    # gaussians that were not relocated are the Adam update alone
    o = 1 / (1 + np.exp(-ref["opacity_raw"].astype(np.float64)))
    kept = o >= np.quantile(o, 0.02)
    np.testing.assert_array_equal(q["color_dc"][kept], ref["color_dc"][kept])
    assert all(np.isfinite(q[k]).all() for k in opipe.PARAM_NAMES)


def test_peer_shards_and_region_layout(pkg):
    """The Adam shards of the peer exchange tile [0, n) in rank order without gaps or overlap,
    each starting on a 16-byte boundary (the device's float4 loads), and the region's four parts
    are 256-byte aligned and disjoint."""
    from tt_splat_b200 import peer
    for n in (1, 3, 4, 5, 59 * 2000 + 1, 59 * 100000 + 1, 5_900_017):
        for world in range(1, 9):
            ranges = [peer.shard_range(n, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (lo, hi), (lo2, _) in zip(ranges, ranges[1:]):
                assert lo <= hi == lo2
            assert all(lo % 4 == 0 for lo, hi in ranges if hi > lo)
    off_p, off_g, off_l, off_f, size = peer.layout(59 * 100000 + 1)
    assert all(o % 256 == 0 for o in (off_p, off_g, off_l, off_f, size))
    assert off_g >= 4 * (59 * 100000 + 1) and off_l >= off_g + 4 * (59 * 100000 + 1)
    assert off_f >= off_l + 4 and size >= off_f + 4 * peer.FLAG_INTS


def test_bench_workload_is_the_baseline_config(pkg):
    """bench.py's headline workload and the synthetic scene it builds are the configuration the
    baseline metric is quoted on (G, image size, K, batch of views, SH degree)."""
    import json
    import os
    import re
    import bench
    from conftest import REPO
    path = os.path.join(REPO, "BASELINE.json")
    if not os.path.exists(path):
        pytest.skip("no baseline description in this checkout")
    text = json.load(open(path))["configs"][2]
    G = int(re.search(r"G=([\d,]+)", text).group(1).replace(",", ""))
    W, H = map(int, re.search(r"(\d+)\s*[x×]\s*(\d+)", text).groups())
    K = int(re.search(r"K=(\d+)", text).group(1))
    views = int(re.search(r"batch of (\d+)", text).group(1))
    deg = int(re.search(r"SH degree (\d+)", text).group(1))
    c = bench.CONFIG
    assert (c["G"], c["W"], c["H"], c["K"], c["views"], c["sh_degree"]) == (G, W, H, K, views, deg)
    sc = pkg.synthetic.config2(G=1000)     # same cameras and images at a small G
    assert len(sc["cams"]) == views and sc["targets"][0].shape == (H, W, 3)
    assert sc["K"] == K and sc["sh_degree"] == deg


def test_status_word_raises_naming_its_bits(pkg, monkeypatch):
    """A bounded device wait that gave up surfaces as a RuntimeError naming the bit: at
    TrainStep.check_status / check_replicas and at the end of fit and train_mcmc (the status
    word is faked here; nothing waits on a device)."""
    from tt_splat_b200 import ops, train
    train.raise_on_status(0)
    with pytest.raises(RuntimeError, match="peer-exchange wait timed out"):
        train.raise_on_status(4)
    with pytest.raises(RuntimeError, match="bulk-copy wait") as e:
        train.raise_on_status(1 | 2 | 64)
    assert "relocation" in str(e.value) and "unknown bits 0x40" in str(e.value)
    st = object.__new__(train.TrainStep)       # host state only: no buffers, no device
    st.dev, st.it, st.pg = torch.device("cpu"), 7, None
    words = [4, 0]
    monkeypatch.setattr(ops, "read_status", lambda: words.pop(0))
    with pytest.raises(RuntimeError, match="iteration 7.*peer-exchange"):
        st.check_replicas()
    st.check_replicas()                          # the read cleared the word: no error


def test_spike_api_refuses_cpu_tensors(pkg):
    """The reference-named functions run kernels only: CPU tensors raise (no CPU fallback)."""
    from tt_splat_b200 import binned, forward, geometry, sh
    z3, z4, z33 = torch.zeros(4, 3), torch.zeros(4, 4), torch.zeros(4, 3, 3)
    calls = [lambda: geometry.quat_to_rotmat(z4), lambda: geometry.cov3d(z3, z33),
             lambda: geometry.project_ewa(z3, z33, torch.eye(3), torch.zeros(3), 1.0, 1.0, 0.0, 0.0),
             lambda: sh.eval_sh_color(3, torch.zeros(4, 16, 3), z3),
             lambda: forward.quad_form(torch.zeros(5), torch.zeros(5), torch.zeros(4, 2), z3),
             lambda: forward.theta_from_conic(z3, torch.zeros(4, 2), 4.0),
             lambda: forward.phi(torch.zeros(5), torch.zeros(5)),
             lambda: forward.quad_form_tilelocal(torch.zeros(5), torch.zeros(5), z3, torch.zeros(4, 2), torch.zeros(2)),
             lambda: forward.poly_splat_wgeo(torch.zeros(5, 4), 4.0),
             lambda: forward.color_from_dc(z3),
             lambda: binned.theta_u_gathered(torch.zeros(2, 4, 3), torch.zeros(2, 4, 2), torch.zeros(2, 2), 4.0)]
    for fn in calls:
        with pytest.raises(RuntimeError, match="CUDA"):
            fn()


def test_camera_conventions(pkg):
    """look_at_opencv, pixel_grid and project_point follow spike/camera.py's conventions: the
    target projects to the principal point, rows are right/down/forward, pixel centres are +0.5
    in row-major order (the OpenGL -> OpenCV pose conversion is pinned bit for bit by the Blender
    loader test against the reference's outputs)."""
    import numpy as np
    from tt_splat_b200 import camera, synthetic
    eye = (1.0, 2.0, -3.5)
    R, t = camera.look_at_opencv(eye, (0.2, -0.1, 0.3))
    Rn, tn = synthetic.look_at_opencv(eye, (0.2, -0.1, 0.3))
    assert np.abs(R.numpy() - Rn).max() < 1e-6 and np.abs(t.numpy() - tn).max() < 1e-6
    assert torch.allclose(R @ R.T, torch.eye(3), atol=1e-6) and abs(float(torch.det(R)) - 1) < 1e-6
    uv, z = camera.project_point(torch.tensor([0.2, -0.1, 0.3]), R, t, 100.0, 90.0, 32.0, 24.0)
    assert torch.allclose(uv, torch.tensor([32.0, 24.0]), atol=1e-4) and float(z) > 0
    uv, _ = camera.project_point(torch.tensor([0.2, -0.1, 0.3]) + R[1], R, t, 100.0, 90.0, 32.0, 24.0)
    assert float(uv[1]) > 24.0                          # +y of the camera is down the image
    px, py = camera.pixel_grid(2, 3)
    assert px.tolist() == [0.5, 1.5, 2.5, 0.5, 1.5, 2.5] and py.tolist() == [0.5, 0.5, 0.5, 1.5, 1.5, 1.5]
    c2w = torch.eye(4)
    c2w[:3, 3] = torch.tensor([0.0, 0.0, 4.0])           # OpenGL camera at +4z looking down -z
    Rv, tv = camera.opengl_c2w_to_opencv_w2c(c2w)
    assert torch.equal(Rv, torch.diag(torch.tensor([1.0, -1.0, -1.0]))) and torch.equal(tv, torch.tensor([0.0, 0.0, 4.0]))


def test_reference_camera_cases(pkg):
    """spike/tests/test_camera.py:16-62 in float64: an OpenGL camera at the origin looks down -z
    (a point in front has z > 0 and lands on the principal point, +x goes right, a point behind
    has z < 0); a camera moved to +4z sees the origin at depth 4; a rotated and translated pose
    gives an orthonormal R_v with determinant 1."""
    from tt_splat_b200 import camera
    f = lambda x: torch.tensor(x, dtype=torch.float64)  # noqa: E731
    fx = fy = 100.0
    cx = cy = 64.0
    R_v, t_v = camera.opengl_c2w_to_opencv_w2c(torch.eye(4, dtype=torch.float64))
    pix, z = camera.project_point(f([0.0, 0.0, -5.0]), R_v, t_v, fx, fy, cx, cy)
    assert z.item() > 0 and torch.allclose(pix, f([cx, cy]), atol=1e-9)
    pix, z = camera.project_point(f([1.0, 0.0, -5.0]), R_v, t_v, fx, fy, cx, cy)
    assert abs(pix[0].item() - (fx / 5.0 + cx)) < 1e-9 and z.item() > 0
    assert camera.project_point(f([0.0, 0.0, 5.0]), R_v, t_v, fx, fy, cx, cy)[1].item() < 0
    c2w = torch.eye(4, dtype=torch.float64)
    c2w[2, 3] = 4.0
    R_v, t_v = camera.opengl_c2w_to_opencv_w2c(c2w)
    pix, z = camera.project_point(f([0.0, 0.0, 0.0]), R_v, t_v, fx, fy, cx, cy)
    assert abs(z.item() - 4.0) < 1e-9 and torch.allclose(pix, f([cx, cy]), atol=1e-9)
    th = 0.5
    c2w = torch.eye(4, dtype=torch.float64)
    c2w[:3, :3] = f([[math.cos(th), 0.0, math.sin(th)], [0.0, 1.0, 0.0], [-math.sin(th), 0.0, math.cos(th)]])
    c2w[:3, 3] = f([1.0, 2.0, 3.0])
    R_v, _ = camera.opengl_c2w_to_opencv_w2c(c2w)
    assert torch.allclose(R_v @ R_v.T, torch.eye(3, dtype=torch.float64), atol=1e-9)
    assert abs(torch.det(R_v).item() - 1.0) < 1e-9


def test_config2_targets_are_8bit(pkg):
    """The headline scene's targets are 8-bit images: the float targets are exactly x / 255 of
    the uint8 ones (what the train step computes on the device from the uploaded bytes)."""
    import numpy as np
    sc = pkg.synthetic.config2(G=500, H=32, W=48, n_views=2)
    for f, u in zip(sc["targets"], sc["targets_u8"]):
        assert u.dtype == np.uint8 and f.dtype == np.float32
        assert np.array_equal(f, u.astype(np.float32) / np.float32(255.0))


def test_32bit_binning_keys_order_like_the_64bit_keys():
    """The warp binning keys (q, stencil offset j, id g) as q<<21 | j<<17 | g when G <= 2^17 and
    (2R+1)^2 <= 16 sort exactly as q<<40 | j<<32 | g, the reference's packed key order (ties in q
    broken by j, then g); every field stays inside its bits."""
    import numpy as np
    rng = np.random.default_rng(0)
    n = 100000
    q = rng.integers(0, 2048, n, dtype=np.uint64)
    q[: n // 4] = 2047                                   # border tiles: many keys tied at the clamp
    j = rng.integers(0, 9, n, dtype=np.uint64)
    g = rng.permutation(1 << 17)[:n].astype(np.uint64)   # unique ids below 2^17
    k64 = (q << np.uint64(40)) | (j << np.uint64(32)) | g
    k32 = ((q << np.uint64(21)) | (j << np.uint64(17)) | g).astype(np.uint32)
    assert int(k32.max()) < 2 ** 32 - 1                 # below the ~0 padding of the warp sort
    assert np.array_equal(np.argsort(k64, kind="stable"), np.argsort(k32, kind="stable"))
    assert np.array_equal(k32 >> np.uint32(21), q.astype(np.uint32))
    assert np.array_equal((k32 >> np.uint32(17)) & np.uint32(15), j.astype(np.uint32))
    assert np.array_equal(k32 & np.uint32((1 << 17) - 1), g.astype(np.uint32))


def _scene_fixture():
    import numpy as np
    from conftest import golden
    z = golden("scene.npz")
    return np, z


@pytest.mark.parametrize("case", [("m_g40", 40, 0.6, 5, True, 0.05), ("m_fresh150", 150, 0.7, 2, False, 0.05),
                                  ("m_gt30", 30, 0.5, 1, True, 0.08), ("m_default4", 4, 1.3, 3, False, 0.05)])
def test_model_draws_equal_the_reference(case, pkg):
    """GaussianModel(G, extent, seed, gt, init_scale) draws the reference's model bit for bit
    (spike/model.py:16-51; tests/golden/make_golden_scene.py)."""
    from tt_splat_b200 import model
    np, z = _scene_fixture()
    name, G, extent, seed, gt, init_scale = case
    m = model.GaussianModel(G, extent=extent, seed=seed, gt=gt, init_scale=init_scale, device="cpu")
    for f in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc"):
        assert np.array_equal(getattr(m, f).detach().numpy(), z[f"{name}__{f}"]), (name, f)


def test_scene_helpers_match_the_reference(pkg):
    """synthetic.make_orbit_cameras and make_gt_model (spike/synthetic.py:16-30): the same camera
    poses and intrinsics as the reference (to float32 rounding), and make_gt_model is the
    reference's gt model."""
    from tt_splat_b200 import synthetic
    np, z = _scene_fixture()
    for name, kw in (("o_default48", dict(n=4, res=48)),
                     ("o_custom", dict(n=3, radius=3.0, elevation=0.2, res=32, fov=0.9))):
        cams = synthetic.make_orbit_cameras(**kw)
        assert np.abs(np.stack([c.R_v.numpy() for c in cams]) - z[f"{name}__R"]).max() < 1e-6
        assert np.abs(np.stack([c.t_v.numpy() for c in cams]) - z[f"{name}__t"]).max() < 1e-5
        k = np.array([[c.fx, c.fy, c.cx, c.cy, c.H, c.W] for c in cams], np.float64)
        assert np.allclose(k, z[f"{name}__k"], rtol=1e-12, atol=0)
    gt = synthetic.make_gt_model(device="cpu")
    assert np.array_equal(gt.means3d.detach().numpy(), z["m_gt30__means3d"])
    assert np.array_equal(gt.color_dc.detach().numpy(), z["m_gt30__color_dc"])
    with pytest.raises(TypeError):
        synthetic.make_gt_model(dtype=torch.float64, device="cpu")


@pytest.mark.parametrize("case", [("p_subset", 500, 200, 11, 7), ("p_pad", 50, 120, 12, 3)])
def test_init_from_points_equals_the_reference(case, pkg):
    """GaussianModel.init_from_points (spike/model.py:55-79) on a seeded cloud with more points
    than gaussians (random subset) and with fewer (jittered copies): means, log-scales and DC
    colours bit for bit."""
    from make_golden_scene import point_cloud
    from tt_splat_b200 import model
    np, z = _scene_fixture()
    name, P, G, cseed, iseed = case
    xyz, rgb = point_cloud(P, cseed)
    m = model.GaussianModel(G, seed=0, device="cpu").init_from_points(xyz, rgb, seed=iseed)
    for f in ("means3d", "log_scales", "color_dc"):
        assert np.array_equal(getattr(m, f).detach().numpy(), z[f"{name}__{f}"]), (name, f)


def test_default_device_is_cuda_or_raises(pkg, monkeypatch):
    """device.default_device (spike/device.py:13-23): CUDA or an error, never a CPU fallback."""
    from tt_splat_b200 import device
    with pytest.raises(ValueError):
        device.default_device("cpu")
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(RuntimeError):
        device.default_device()
    with pytest.raises(RuntimeError):
        device.default_device("cuda:0")
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    assert device.default_device() == torch.device("cuda")
    assert device.default_device("cuda:1") == torch.device("cuda", 1)
