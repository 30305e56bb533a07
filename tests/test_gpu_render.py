"""Fused per-tile forward/backward and the full render pipeline vs the reference and the oracle.
Tolerances (north star): images 1e-3 max abs in fp32 (bf16 slot rows 1e-2), gradients 1e-3
relative L2."""
import numpy as np
import pytest
import torch

from conftest import cam_from, golden, params_from, rel_l2
from oracle import binning, pipeline, render as orender

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_render_on_reference_operands(pkg):
    """_DevRenderBinned on the reference's own operands reproduces its image and operand grads."""
    from tt_splat_b200 import binned
    z = golden("render_config0.npz")
    cam = cam_from(z)
    tm = binned.TileMap(cam["H"], cam["W"])
    th = torch.from_numpy(z["theta_u"]).to(DEV).requires_grad_(True)
    col = torch.from_numpy(z["col"]).to(DEV).requires_grad_(True)
    oc = torch.from_numpy(z["oc"]).to(DEV).requires_grad_(True)
    wb = torch.tensor(float(z["w_b"]), device=DEV, requires_grad=True)
    img = binned._DevRenderBinned.apply(th, col, oc, wb, tm.Phi, tm.gidx, torch.ones(3, device=DEV), cam["H"], cam["W"])
    assert np.abs(img.detach().cpu().numpy() - z["img"]).max() < 1e-4
    tgt = torch.from_numpy(z["target"]).to(DEV)
    (img - tgt).abs().mean().backward()
    assert rel_l2(th.grad.cpu().numpy(), z["gtheta"]) < 1e-4
    assert rel_l2(col.grad.cpu().numpy(), z["gcol"]) < 1e-4
    assert rel_l2(oc.grad.cpu().numpy(), z["goc"]) < 1e-4
    assert abs(float(wb.grad) - float(z["gw_b"])) < 1e-4 * abs(float(z["gw_b"]))


def _model(pkg, p):
    return pkg.model.GaussianModel.from_arrays(p, device=DEV)


@pytest.mark.parametrize("fixture,deg", [("render_config0.npz", 0), ("render_sh3.npz", 3)])
def test_pipeline_vs_reference_and_oracle(fixture, deg, pkg):
    from tt_splat_b200 import camera, render
    z = golden(fixture)
    cam = cam_from(z)
    p = params_from(z)
    K = int(z["K"])
    m = _model(pkg, p)
    img = render.render(m, camera.Camera.from_dict(cam), "A", sh_degree=deg, K=K)
    fw = pipeline.render_view(p, deg, cam, K=K)
    out = img.detach().cpu().numpy()
    assert np.abs(out - fw["img"]).max() < 1e-3
    assert np.abs(out - z["img"]).max() < 1e-3
    tgt = torch.from_numpy(z["target"]).to(DEV)
    (img - tgt).abs().mean().backward()
    g = m.flat.grad
    G = p["means3d"].shape[0]
    from tt_splat_b200.model import view
    gimg = (np.sign(fw["img"] - z["target"]) / fw["img"].size).astype(np.float32)
    go = pipeline.backward_view(fw, gimg, p, deg)
    names = ["means3d", "log_scales", "quats", "opacity_raw", "color_dc"] + (["color_rest"] if deg else [])
    for n in names:
        mine = view(g, G, n).cpu().numpy()
        assert rel_l2(mine, z["grad_" + n]) < 1e-3, (n, rel_l2(mine, z["grad_" + n]))
        assert rel_l2(mine, go[n]) < 1e-3, (n, rel_l2(mine, go[n]))
    assert abs(float(view(g, G, "w_b_raw")) - float(z["grad_w_b_raw"])) < 1e-3 * abs(float(z["grad_w_b_raw"]))


@pytest.mark.parametrize("deg", [0, 3])
def test_arm_b_vs_reference_and_oracle(deg, pkg):
    """Arm B: image and gradients (the two depth parameters included) against the reference's dense
    render + autograd and against the oracle."""
    from tt_splat_b200 import camera, render
    from tt_splat_b200.model import view
    z = golden("render_arm_b.npz")
    cam = cam_from(z)
    p = params_from(z)
    K = int(z["K"])
    m = _model(pkg, p)
    with torch.no_grad():
        m.depth_beta.fill_(float(z["depth_beta"]))
        m.depth_tau.fill_(float(z["depth_tau"]))
    img = render.render(m, camera.Camera.from_dict(cam), "B", sh_degree=deg, K=K)
    fw = pipeline.render_view(p, deg, cam, K=K, depth_bt=(float(z["depth_beta"]), float(z["depth_tau"])))
    pre = f"deg{deg}__"
    out = img.detach().cpu().numpy()
    assert np.abs(out - z[pre + "img"]).max() < 1e-3
    assert np.abs(out - fw["img"]).max() < 1e-3
    wts = z["wts"].astype(np.float32)
    (img * torch.from_numpy(wts).to(DEV)).sum().backward()
    go = pipeline.backward_view(fw, wts, p, deg)
    G = p["means3d"].shape[0]
    g = m.flat.grad
    names = ["means3d", "log_scales", "quats", "opacity_raw", "color_dc"] + (["color_rest"] if deg else [])
    for n in names:
        mine = view(g, G, n).cpu().numpy()
        assert rel_l2(mine, z[pre + "grad_" + n]) < 1e-3, (n, rel_l2(mine, z[pre + "grad_" + n]))
        assert rel_l2(mine, go[n]) < 1e-3, (n, rel_l2(mine, go[n]))
    mine = {"w_b_raw": float(view(g, G, "w_b_raw")), "depth_beta": float(m.depth_beta.grad),
            "depth_tau": float(m.depth_tau.grad)}
    for n, v in mine.items():
        ref = float(z[pre + "grad_" + n])
        assert abs(v - ref) < 1e-3 * abs(ref), (n, v, ref)
    # arm A ignores the depth parameters
    m.flat.grad = None
    m.depth_beta.grad = None
    render.render(m, camera.Camera.from_dict(cam), "A", sh_degree=deg, K=K).sum().backward()
    assert m.depth_beta.grad is None or float(m.depth_beta.grad) == 0.0


@pytest.mark.parametrize("deg", [0, 3])
def test_arm_rv_vs_reference_and_oracle(deg, pkg):
    """Arm RV (revealage compositing): image and gradients against the reference's dense render +
    autograd and against the oracle; six pixels carry weights above the clamp bound."""
    from tt_splat_b200 import camera, render
    from tt_splat_b200.model import view
    z = golden("render_arm_rv.npz")
    cam = cam_from(z)
    p = params_from(z)
    K = int(z["K"])
    m = _model(pkg, p)
    img = render.render(m, camera.Camera.from_dict(cam), "RV", sh_degree=deg, K=K)
    fw = pipeline.render_view(p, deg, cam, K=K, arm="RV")
    pre = f"deg{deg}__"
    out = img.detach().cpu().numpy()
    assert np.abs(out - z[pre + "img"]).max() < 1e-3
    assert np.abs(out - fw["img"]).max() < 1e-3
    wts = z["wts"].astype(np.float32)
    (img * torch.from_numpy(wts).to(DEV)).sum().backward()
    go = pipeline.backward_view(fw, wts, p, deg)
    G = p["means3d"].shape[0]
    g = m.flat.grad
    names = ["means3d", "log_scales", "quats", "opacity_raw", "color_dc"] + (["color_rest"] if deg else [])
    for n in names:
        mine = view(g, G, n).cpu().numpy()
        assert rel_l2(mine, z[pre + "grad_" + n]) < 1e-3, (n, rel_l2(mine, z[pre + "grad_" + n]))
        assert rel_l2(mine, go[n]) < 1e-3, (n, rel_l2(mine, go[n]))
    assert float(view(g, G, "w_b_raw")) == 0.0
    with pytest.raises(NotImplementedError):
        render.render(m, camera.Camera.from_dict(cam), "RV", sh_degree=deg, K=K, bf16=True)


def test_near_plane_needles_stay_finite_and_match_float64(pkg):
    """The near-plane needles of geom_near_plane.npz (the reference's fp32 conic clamps to ~1e20
    for half of them): the fused projection's conics are within 1e-3 of the float64 oracle, and a
    1264x832 render of a scene containing them is finite and matches the oracle's binned render."""
    from tt_splat_b200 import camera, ops, render
    from tt_splat_b200.model import pack_arrays
    from oracle import geometry as ogeom
    z = golden("geom_near_plane.npz")
    cam = cam_from(z)
    n = z["means3d"].shape[0]
    needles = dict(means3d=z["means3d"], log_scales=z["log_scales"], quats=z["quats"],
                   opacity_raw=np.zeros(n, np.float32), color_dc=np.zeros((n, 3), np.float32),
                   color_rest=np.zeros((n, 15, 3), np.float32))
    scene = pkg.synthetic.config2(seed=21, G=3000, n_views=1)["params"]
    p = {k: np.concatenate([scene[k], needles[k]]) for k in needles}
    p["w_b_raw"] = scene["w_b_raw"]
    G = p["means3d"].shape[0]
    flat = pack_arrays(p).to(DEV)
    cams_t = camera.pack_cameras([camera.Camera.from_dict(cam)], DEV)
    pj = ops.project(flat, G, 3, cams_t, cam["H"], cam["W"])
    dev_conic = pj["proj"][0, G - n:, 2:5].cpu().numpy()
    conic64, _, _, _, _ = ogeom.fwd(z["means3d"], z["quats"], z["log_scales"], cam)
    assert np.abs(dev_conic - conic64).max() / np.abs(conic64).max() < 1e-3
    img = render.render(_model(pkg, p), camera.Camera.from_dict(cam), "A", sh_degree=3).detach().cpu().numpy()
    assert np.isfinite(img).all()
    ref = pipeline.render_view(p, 3, cam)["img"]
    assert np.abs(img - ref).max() < 1e-3


@pytest.mark.parametrize("deg", [1, 2])
def test_sh_degree_1_2_vs_reference(deg, pkg):
    """The device path at SH degrees 1 and 2: image and gradients against the reference."""
    from tt_splat_b200 import camera, render
    from tt_splat_b200.model import view
    z = golden("render_sh12.npz")
    cam = cam_from(z)
    p = params_from(z)
    m = _model(pkg, p)
    img = render.render(m, camera.Camera.from_dict(cam), "A", sh_degree=deg, K=int(z["K"]))
    pre = f"deg{deg}__"
    assert np.abs(img.detach().cpu().numpy() - z[pre + "img"]).max() < 1e-3
    (img * torch.from_numpy(z["wts"].astype(np.float32)).to(DEV)).sum().backward()
    G = p["means3d"].shape[0]
    for n in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest"):
        mine = view(m.flat.grad, G, n).cpu().numpy()
        assert rel_l2(mine, z[pre + "grad_" + n]) < 1e-3, (n, rel_l2(mine, z[pre + "grad_" + n]))
    ref = float(z[pre + "grad_w_b_raw"])
    assert abs(float(view(m.flat.grad, G, "w_b_raw")) - ref) < 1e-3 * abs(ref)


def test_operator_pair_vs_reference(pkg):
    """The reference's operator pair (_operands + _DevRenderBinned via render_binned_device,
    tools/m4_train_binned.py:189-219): tables, image and parameter gradients."""
    from tt_splat_b200 import binned, camera
    from tt_splat_b200.model import view
    z = golden("render_config0.npz")
    cam = cam_from(z)
    p = params_from(z)
    m = _model(pkg, p)
    tmap = binned.TileMap(cam["H"], cam["W"])
    img, (idx, valid) = binned.render_binned_device(m, camera.Camera.from_dict(cam), tmap, K=int(z["K"]),
                                                    return_bins=True)
    v = valid.cpu().numpy()
    assert np.array_equal(np.where(v, idx.cpu().numpy(), -1), np.where(z["valid"], z["idx"], -1))
    assert np.abs(img.detach().cpu().numpy() - z["img"]).max() < 1e-3
    tgt = torch.from_numpy(z["target"]).to(DEV)
    (img - tgt).abs().mean().backward()
    G = p["means3d"].shape[0]
    for n in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc"):
        mine = view(m.flat.grad, G, n).cpu().numpy()
        assert rel_l2(mine, z["grad_" + n]) < 1e-3, (n, rel_l2(mine, z["grad_" + n]))


def test_operator_pair_cached_bins(pkg):
    """cached_bins (tools/m4_train_binned.py:203-207): the same tables at the same parameters give
    the same image and gradients; stale tables after the means moved match the oracle driven by
    those tables."""
    import types
    from tt_splat_b200 import binned, camera
    from tt_splat_b200.model import view
    z = golden("render_config0.npz")
    cam = cam_from(z)
    c = camera.Camera.from_dict(cam)
    p = params_from(z)
    K = int(z["K"])
    G = p["means3d"].shape[0]
    tmap = binned.TileMap(cam["H"], cam["W"])
    m = _model(pkg, p)
    img0, bins = binned.render_binned_device(m, c, tmap, K=K, return_bins=True)
    img0.sum().backward()
    g0 = m.flat.grad.clone()
    m.flat.grad = None
    img1, bins1 = binned.render_binned_device(m, c, tmap, K=K, cached_bins=bins, return_bins=True)
    assert bins1 is bins
    assert torch.equal(img1, img0)
    img1.sum().backward()
    assert rel_l2(m.flat.grad.cpu().numpy(), g0.cpu().numpy()) < 1e-6
    # stale tables: move the means by up to a third of a tile, re-render through the old tables
    p1 = dict(p)
    p1["means3d"] = (p["means3d"] + 0.02 * np.random.default_rng(3).standard_normal(p["means3d"].shape)).astype(np.float32)
    m1 = _model(pkg, p1)
    img, _ = binned.render_binned_device(m1, c, tmap, K=K, cached_bins=bins, return_bins=True)
    tb = types.SimpleNamespace(idx=bins[0].cpu().numpy(), valid=bins[1].cpu().numpy())
    fw = pipeline.render_view(p1, 0, cam, K=K, bins=tb)
    assert np.abs(img.detach().cpu().numpy() - fw["img"]).max() < 1e-3
    wts = np.random.default_rng(4).standard_normal(fw["img"].shape).astype(np.float32)
    (img * torch.from_numpy(wts).to(DEV)).sum().backward()
    go = pipeline.backward_view(fw, wts, p1, 0)
    for n in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc"):
        mine = view(m1.flat.grad, G, n).cpu().numpy()
        assert rel_l2(mine, go[n]) < 1e-3, (n, rel_l2(mine, go[n]))
    from tt_splat_b200 import ops
    assert ops.read_status() == 0
    bad = (bins[0].clone(), bins[1].clone())
    bad[1][0, 0] = False                        # a hole before valid slots
    with pytest.raises(ValueError):
        binned.render_binned_device(m, c, tmap, K=K, cached_bins=bad)


def test_slot_rows_bit_exact_given_projection(pkg):
    """theta_u rows of the pack epilogue are the reference's fp32 expression bit for bit,
    given the device's own mu2d/conic (tools/m4_train_binned.py:130-143)."""
    from tt_splat_b200 import camera, ops
    from tt_splat_b200.model import pack_arrays
    sc = pkg.synthetic.config0(seed=3, G=1500, res=96)
    flat = pack_arrays(sc["params"]).to(DEV)
    cams = camera.pack_cameras([camera.Camera.from_dict(sc["cams"][0])], DEV)
    pj = ops.project(flat, 1500, 0, cams, 96, 96)
    bp = ops.bin_pack(pj, 1500, 96, 96, 1, 64)
    proj = pj["proj"][0].cpu().numpy()
    idx = bp["idx"][0].cpu().numpy()
    valid = idx >= 0
    tm = binning.tile_map(96, 96)
    ii = np.where(valid, idx, 0)
    th = orender.theta_u_gathered(proj[ii][..., 2:5], proj[ii][..., 0:2], tm.origins, 4.0) * valid[:, None, :]
    rows = bp["slots"][0].cpu().numpy()
    assert np.array_equal(np.transpose(rows[..., :6], (0, 2, 1))[np.broadcast_to(valid[:, None, :], th.shape)],
                          th[np.broadcast_to(valid[:, None, :], th.shape)])
    assert np.array_equal(rows[..., 6:9][valid], proj[ii][..., 5:8][valid])


def test_bf16_slot_rows(pkg):
    """bf16 operands, fp32 accumulation, against the oracle's image: north_star's 1e-2 bound
    (max abs) and the relative-L2 metric the reference reports for its bf16 device path
    (tools/m4_train_binned.py:246-248).  The compact rows carry theta_u as a bf16 (hi, lo) pair,
    colour_o and o_col as bf16."""
    from tt_splat_b200 import camera, render
    sc = pkg.synthetic.config1(seed=4, G=3000, res=128)
    m = _model(pkg, sc["params"])
    cam = camera.Camera.from_dict(sc["cams"][0])
    ref = pipeline.render_view(sc["params"], 3, sc["cams"][0], K=128)["img"]
    with torch.no_grad():
        b = render.render(m, cam, sh_degree=3, bf16=True)
    c = render.render(m, cam, sh_degree=3, bf16=True)          # with grad: fp32 rows kept for backward
    assert np.abs(b.cpu().numpy() - ref).max() < 1e-2
    assert rel_l2(b.cpu().numpy(), ref) < 1e-3
    assert torch.equal(b, c.detach())


def test_compact_bf16_rows_reconstruct_theta(pkg):
    """theta_hi + theta_lo reproduces the fp32 theta_u to ~2^-16 relative; colour_o and o_col are
    the fp32 values rounded to bf16."""
    from tt_splat_b200 import camera, ops
    from tt_splat_b200.model import pack_arrays
    sc = pkg.synthetic.config1(seed=6, G=4000, res=128)
    flat = pack_arrays(sc["params"]).to(DEV)
    cams = camera.pack_cameras([camera.Camera.from_dict(sc["cams"][0])], DEV)
    pj = ops.project(flat, 4000, 3, cams, 128, 128)
    f = ops.bin_pack(pj, 4000, 128, 128, 1, 128)
    h = ops.bin_pack(pj, 4000, 128, 128, 1, 128, with_inv=False, bf16=True)
    assert torch.equal(f["idx"], h["idx"]) and torch.equal(f["count"], h["count"])
    valid = (f["idx"] >= 0)[..., None]
    rf = f["slots"].float()
    rh = h["slots"].float()
    theta = rh[..., 0:6] + rh[..., 6:12]
    err = ((theta - rf[..., 0:6]).abs() / rf[..., 0:6].abs().clamp(min=1e-30))[valid.expand_as(theta)]
    assert float(err.max()) < 2.0 ** -15
    assert torch.equal(rh[..., 12:16][valid.expand(-1, -1, -1, 4)],
                       rf[..., 6:10].to(torch.bfloat16).float()[valid.expand(-1, -1, -1, 4)])


def test_multi_view_batch_equals_single_views(pkg):
    from tt_splat_b200 import camera, render
    sc = pkg.synthetic.config2(seed=5, G=5000, H=64, W=96, n_views=3)
    m = _model(pkg, sc["params"])
    cams = [camera.Camera.from_dict(c) for c in sc["cams"]]
    batch = render.render_views(m, cams, sh_degree=3).detach()
    for v, c in enumerate(cams):
        assert torch.equal(batch[v], render.render(m, c, sh_degree=3).detach())


def test_dense_wsr_polysplat_vs_oracle(pkg):
    from tt_splat_b200 import backward
    rng = np.random.default_rng(0)
    G, P = 37, 300
    th = rng.standard_normal((G, 6)).astype(np.float32) * np.array([0.02, 0.02, 0.02, 0.3, 0.3, 0.5], np.float32)
    th[:, 5] += 0.5
    o = rng.uniform(0.1, 0.9, G).astype(np.float32)
    col = rng.uniform(0, 1, (G, 3)).astype(np.float32)
    px = rng.uniform(0, 16, P)
    py = rng.uniform(0, 16, P)
    Phi = np.stack([px * px, py * py, px * py, px, py, np.ones(P)], -1).astype(np.float32)
    keep = (rng.random(G) > 0.2).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV).requires_grad_(True)  # noqa: E731
    tth, to, tcol = t(th), t(o), t(col)
    wb = torch.tensor(0.05, device=DEV, requires_grad=True)
    C = backward.wsr_polysplat(tth, to, tcol, wb, t(Phi).detach(), torch.ones(3, device=DEV), t(keep).detach())
    ref = orender.wsr_dense_fwd(th, o, col, 0.05, Phi, np.ones(3), keep)
    assert np.abs(C.detach().cpu().numpy() - ref).max() < 1e-5
    gC = rng.standard_normal((P, 3)).astype(np.float32)
    C.backward(torch.from_numpy(gC).to(DEV))
    gth, go, gcol, gwb = orender.wsr_dense_bwd(gC, th, o, col, 0.05, Phi, np.ones(3), keep)
    assert rel_l2(tth.grad.cpu().numpy(), gth) < 1e-4
    assert rel_l2(to.grad.cpu().numpy(), go) < 1e-4
    assert rel_l2(tcol.grad.cpu().numpy(), gcol) < 1e-4
    assert abs(float(wb.grad) - gwb) < 1e-4 * abs(gwb)


def test_dead_slots_change_no_bits(pkg):
    """Slots whose weight is zero at every pixel of their tile (u <= 0 everywhere: gaussians
    binned into neighbouring tiles they never reach) are skipped by the tile kernels.  Removing
    the clearly dead ones from the tables (max u <= -1e-3) leaves the image, the denominators, the
    live slots' gradients and the w_b partials bit for bit unchanged, and the removed slots'
    gradients are exactly zero."""
    from tt_splat_b200 import ops
    from tt_splat_b200.model import pack_arrays
    from tt_splat_b200 import camera
    sc = pkg.synthetic.config2(seed=13, G=6000, H=96, W=128, n_views=2)
    G, H, W = 6000, 96, 128
    flat = pack_arrays(sc["params"]).to(DEV)
    cams = camera.pack_cameras([camera.Camera.from_dict(c) for c in sc["cams"]], DEV)
    pj = ops.project(flat, G, 3, cams, H, W)
    bp = ops.bin_pack(pj, G, H, W, 1, 64)
    slots, count = bp["slots"], bp["count"]
    V, T, K, _ = slots.shape
    c_b = torch.ones(3, device=DEV)
    p = torch.arange(16, device=DEV, dtype=torch.float32) + 0.5
    py, px = torch.meshgrid(p, p, indexing="ij")
    phi = torch.stack([px * px, py * py, px * py, px, py, torch.ones_like(px)], -1).reshape(256, 6)
    umax = torch.einsum("vtkc,pc->vtkp", slots[..., :6], phi).amax(-1)
    valid = torch.arange(K, device=DEV)[None, None, :] < count[..., None]
    keep = valid & (umax > -1e-3)
    assert int((valid & ~keep).sum()) > 0                      # the scene has dead slots
    # compacted tables: the kept slots of each tile first, in order
    order = torch.argsort((~keep).to(torch.int8), dim=-1, stable=True)
    slots2 = torch.gather(slots, 2, order[..., None].expand(-1, -1, -1, slots.shape[-1])).contiguous()
    count2 = keep.sum(-1).to(torch.int32).contiguous()
    a = ops.render_fwd(slots, count, H, W, flat[59 * G:], c_b)
    b = ops.render_fwd(slots2, count2, H, W, flat[59 * G:], c_b)
    assert torch.equal(a["img"], b["img"]) and torch.equal(a["den"], b["den"])
    gimg = torch.randn(a["img"].shape, device=DEV, generator=torch.Generator(DEV).manual_seed(2))
    ga = ops.render_bwd(slots, count, H, W, c_b, a["img"], a["den"], gimg)
    gb = ops.render_bwd(slots2, count2, H, W, c_b, b["img"], b["den"], gimg)
    assert torch.equal(ga["gwb"], gb["gwb"])
    kept_a = torch.gather(ga["slot_grads"], 2, order[..., None].expand(-1, -1, -1, 10))
    live2 = torch.arange(K, device=DEV)[None, None, :] < count2[..., None]
    assert torch.equal(kept_a[live2], gb["slot_grads"][live2])
    assert (ga["slot_grads"][valid & ~keep] == 0).all()


def test_dead_slots_without_inverse_entries_change_no_bits(pkg):
    """With fp32 slot rows the binning leaves dead slots out of the inverse table; the parameter
    backward through it equals, bit for bit, the one through the complete table of the same
    binning, and the entries left out are exactly the dead-marked slots'."""
    from tt_splat_b200 import camera, ops
    from tt_splat_b200.model import pack_arrays
    sc = pkg.synthetic.config2(seed=14, G=6000, H=96, W=128, n_views=2)
    G, H, W, K = 6000, 96, 128, 64
    flat = pack_arrays(sc["params"]).to(DEV)
    cams = camera.pack_cameras([camera.Camera.from_dict(c) for c in sc["cams"]], DEV)
    pj = ops.project(flat, G, 3, cams, H, W)
    bp = ops.bin_pack(pj, G, H, W, 1, K)
    full = ops.bin_from_mu2d(pj["mu2d"], pj["keep"], H, W, 1, K)       # no rows: complete table
    assert torch.equal(bp["idx"], full[0])
    inv_p, inv_f = bp["inv"], full[3]
    dead = bp["slots"][..., 10] != 0
    valid = bp["idx"] >= 0
    assert int((dead & valid).sum()) > 0
    flatpos = torch.arange(bp["idx"][0].numel(), device=DEV).reshape(bp["idx"].shape[1:])
    for v in range(2):
        dead_pos = set(flatpos[dead[v] & valid[v]].tolist())
        missing = (inv_f[v] >= 0) & (inv_p[v] < 0)
        assert set(inv_f[v][missing].tolist()) == dead_pos
        assert torch.equal(inv_p[v][inv_p[v] >= 0], inv_f[v][inv_p[v] >= 0])
    c_b = torch.ones(3, device=DEV)
    rf = ops.render_fwd(bp["slots"], bp["count"], H, W, flat[59 * G:], c_b)
    gimg = torch.randn(rf["img"].shape, device=DEV, generator=torch.Generator(DEV).manual_seed(4))
    rb = ops.render_bwd(bp["slots"], bp["count"], H, W, c_b, rf["img"], rf["den"], gimg)
    ga = ops.backward_params(flat, G, 3, cams, H, W, 1, K, inv_p, rb["slot_grads"], rb["gwb"], proj=pj["proj"])
    gb = ops.backward_params(flat, G, 3, cams, H, W, 1, K, inv_f, rb["slot_grads"], rb["gwb"], proj=pj["proj"])
    assert torch.equal(ga, gb)
