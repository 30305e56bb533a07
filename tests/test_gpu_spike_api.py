"""The composable spike API on the device: every function of spike/geometry.py, spike/sh.py and
spike/forward.py that this package exports runs a kernel forward and a kernel backward.

Each is checked against the oracle (float64 restatement of the reference, pinned to the
reference's fixtures) at 1e-12 in float64 and 1e-5 in float32, its backward against torch's
finite-difference gradcheck in float64, and the composed geometry chain against the reference's
own fixture (tests/golden/geom_bwd.npz, written by tools/geom_bwd.py): conic and mean values and
the gradients of means, quaternions and log-scales.
"""
import numpy as np
import pytest
import torch

from conftest import cam_from, golden, rel_l2
from oracle import geometry as ogeom
from oracle import sh as osh

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(x, dt=torch.float64, grad=False):
    return torch.tensor(np.asarray(x), dtype=dt, device=DEV).requires_grad_(grad)


def _scene(seed=0, G=64):
    rng = np.random.default_rng(seed)
    means = rng.uniform(-1, 1, (G, 3))
    quats = rng.standard_normal((G, 4))
    ls = rng.normal(-2.0, 0.4, (G, 3))
    cam = dict(R_v=np.eye(3), t_v=np.array([0.1, -0.2, 4.0]), fx=300.0, fy=310.0, cx=64.0, cy=60.0)
    return means, quats, ls, cam


def test_quat_cov_project_vs_oracle():
    from tt_splat_b200 import geometry
    means, quats, ls, cam = _scene()
    for dt, tol in ((torch.float64, 1e-12), (torch.float32, 1e-5)):
        R = geometry.quat_to_rotmat(_t(quats, dt))
        assert rel_l2(R.cpu().numpy(), ogeom.quat_to_rotmat(quats)) < tol
        cov = geometry.cov3d(torch.exp(_t(ls, dt)), R)
        cov_ref = ogeom.cov3d(np.exp(ls), ogeom.quat_to_rotmat(quats))
        assert rel_l2(cov.cpu().numpy(), cov_ref) < tol
        mu2d, conic, depth, keep = geometry.project_ewa(_t(means, dt), cov, torch.tensor(cam["R_v"], dtype=dt),
                                                        torch.tensor(cam["t_v"], dtype=dt), cam["fx"], cam["fy"],
                                                        cam["cx"], cam["cy"])
        m_ref, c_ref, d_ref, k_ref = ogeom.project_ewa(means, cov_ref, cam["R_v"], cam["t_v"], cam["fx"], cam["fy"],
                                                       cam["cx"], cam["cy"])
        assert keep.dtype == torch.bool and np.array_equal(keep.cpu().numpy(), k_ref)
        assert rel_l2(mu2d.detach().cpu().numpy(), m_ref) < tol
        assert rel_l2(conic.detach().cpu().numpy(), c_ref) < 10 * tol
        assert rel_l2(depth.detach().cpu().numpy(), d_ref) < tol


def test_geometry_gradcheck():
    from tt_splat_b200 import geometry
    means, quats, ls, cam = _scene(1, G=12)
    means[0, 2] = -4.05                      # one gaussian behind the near plane (z clamp)
    q = _t(quats, grad=True)
    assert torch.autograd.gradcheck(geometry.quat_to_rotmat, (q,))
    s = _t(np.exp(ls), grad=True)
    R = _t(ogeom.quat_to_rotmat(quats), grad=True)
    assert torch.autograd.gradcheck(geometry.cov3d, (s, R))
    Rv, tv = torch.tensor(cam["R_v"]), torch.tensor(cam["t_v"])

    def proj(m, c):
        mu, con, d, _ = geometry.project_ewa(m, c, Rv, tv, cam["fx"], cam["fy"], cam["cx"], cam["cy"])
        return mu, con, d
    cov = _t(ogeom.cov3d(np.exp(ls), ogeom.quat_to_rotmat(quats)), grad=True)
    assert torch.autograd.gradcheck(proj, (_t(means, grad=True), cov))


def test_geometry_chain_vs_reference_fixture():
    """quat_to_rotmat -> cov3d -> project_ewa on the device (float32) against the reference's
    tools/geom_bwd.py outputs and gradients for the fixture's random output gradients."""
    from tt_splat_b200 import geometry
    z = golden("geom_bwd.npz")
    cam = cam_from(z)
    m = _t(z["means3d"], torch.float32, True)
    q = _t(z["quats"], torch.float32, True)
    ls = _t(z["log_scales"], torch.float32, True)
    cov = geometry.cov3d(torch.exp(ls), geometry.quat_to_rotmat(q))
    mu2d, conic, _, keep = geometry.project_ewa(m, cov, torch.from_numpy(cam["R_v"]), torch.from_numpy(cam["t_v"]),
                                                cam["fx"], cam["fy"], cam["cx"], cam["cy"])
    assert rel_l2(conic.detach().cpu().numpy(), z["conic"]) < 1e-5
    assert rel_l2(mu2d.detach().cpu().numpy(), z["mu2d"]) < 1e-6
    ((conic * _t(z["gconic"], torch.float32)).sum() + (mu2d * _t(z["gmu"], torch.float32)).sum()).backward()
    assert rel_l2(m.grad.cpu().numpy(), z["gmeans"]) < 1e-4
    assert rel_l2(q.grad.cpu().numpy(), z["gquats"]) < 1e-4
    assert rel_l2(ls.grad.cpu().numpy(), z["glog_scales"]) < 1e-4


@pytest.mark.parametrize("deg", [0, 1, 2, 3])
def test_eval_sh_color_vs_oracle(deg):
    from tt_splat_b200 import sh
    rng = np.random.default_rng(deg)
    G = 200
    coeffs = rng.normal(0, 0.4, (G, 16, 3))
    coeffs[:, 0] = rng.uniform(-2, 2, (G, 3))         # some colours clamp at zero
    dirs = rng.standard_normal((G, 3))
    ref, _ = osh.eval_sh_color(deg, coeffs, dirs)
    c, d = _t(coeffs, grad=True), _t(dirs, grad=True)
    out = sh.eval_sh_color(deg, c, d)
    assert np.abs(out.detach().cpu().numpy() - ref).max() < 1e-12
    g = rng.standard_normal((G, 3))
    out.backward(_t(g))
    gco, gd = osh.eval_sh_color_bwd(deg, coeffs, dirs, g)
    nb = (deg + 1) ** 2
    assert np.abs(c.grad.cpu().numpy()[:, :nb] - gco).max() < 1e-12
    assert (c.grad.cpu().numpy()[:, nb:] == 0).all()
    assert np.abs(d.grad.cpu().numpy() - gd).max() < 1e-10
    out32 = sh.eval_sh_color(deg, _t(coeffs, torch.float32), _t(dirs, torch.float32))
    assert np.abs(out32.cpu().numpy() - ref).max() < 1e-5
    cs, ds = _t(coeffs[:8], grad=True), _t(dirs[:8], grad=True)
    assert torch.autograd.gradcheck(lambda a, b: sh.eval_sh_color(deg, a, b), (cs, ds))


def test_forward_primitives_vs_numpy_and_gradcheck():
    from tt_splat_b200 import forward
    rng = np.random.default_rng(3)
    P, G = 50, 9
    px, py = rng.uniform(0, 32, P), rng.uniform(0, 32, P)
    mu = rng.uniform(0, 32, (G, 2))
    A = rng.standard_normal((G, 2, 2))
    S = A @ np.swapaxes(A, 1, 2) + 0.5 * np.eye(2)
    conic = np.stack([S[:, 0, 0], S[:, 0, 1], S[:, 1, 1]], 1) * 0.05
    dx, dy = px[:, None] - mu[None, :, 0], py[:, None] - mu[None, :, 1]
    Q_ref = conic[:, 0] * dx * dx + 2 * conic[:, 1] * dx * dy + conic[:, 2] * dy * dy
    Q = forward.quad_form(_t(px), _t(py), _t(mu), _t(conic))
    assert np.abs(Q.cpu().numpy() - Q_ref).max() < 1e-10 * np.abs(Q_ref).max()
    # the monomial identity Q = Phi theta_Q^T (spike/tests/test_transform.py:15-31)
    thQ, thU = forward.theta_from_conic(_t(conic), _t(mu), 4.0)
    Phi = forward.phi(_t(px), _t(py))
    assert np.abs((Phi @ thQ.T).cpu().numpy() - Q_ref).max() < 1e-9 * np.abs(Q_ref).max()
    assert np.abs((Phi @ thU.T).cpu().numpy() - (1 - Q_ref / 4.0)).max() < 1e-9 * np.abs(Q_ref).max()
    # tile-local GEMM form equals the global form
    org = np.array([16.0, 8.0])
    Qt = forward.quad_form_tilelocal(_t(px - org[0]), _t(py - org[1]), _t(conic), _t(mu), _t(org))
    assert np.abs(Qt.cpu().numpy() - Q_ref).max() < 1e-9 * np.abs(Q_ref).max()
    keep = torch.tensor(rng.random(G) > 0.3, device=DEV)
    w = forward.poly_splat_wgeo(_t(Q_ref), 4.0, keep)
    w_ref = np.maximum(0, 1 - Q_ref / 4.0) ** 2 * keep.cpu().numpy()[None, :]
    assert np.abs(w.cpu().numpy() - w_ref).max() < 1e-12
    dc = rng.normal(0, 2, (G, 3))
    assert np.abs(forward.color_from_dc(_t(dc)).cpu().numpy() - np.maximum(0.5 + osh.C0 * dc, 0)).max() < 1e-12
    # backward of every primitive against finite differences (float64)
    tp, tq, tm, tc = _t(px), _t(py), _t(mu, grad=True), _t(conic, grad=True)
    assert torch.autograd.gradcheck(lambda m, c: forward.quad_form(tp, tq, m, c), (tm, tc))
    assert torch.autograd.gradcheck(lambda c, m: forward.theta_from_conic(c, m, 4.0), (tc, tm))
    assert torch.autograd.gradcheck(forward.phi, (_t(px[:8], grad=True), _t(py[:8], grad=True)))
    assert torch.autograd.gradcheck(
        lambda c, m: forward.quad_form_tilelocal(_t(px[:8] - 16), _t(py[:8] - 8), c, m, _t(org)), (tc, tm))
    qv = _t(Q_ref[:6] + 0.01, grad=True)
    assert torch.autograd.gradcheck(lambda q: forward.poly_splat_wgeo(q, 4.0, keep), (qv,))
    assert torch.autograd.gradcheck(forward.color_from_dc, (_t(dc[:4] + 0.05, grad=True),))


def test_theta_u_gathered_matches_slot_rows(pkg):
    """binned.theta_u_gathered (the [T,6,K] operand, tools/m4_train_binned.py:130-143) on the
    device equals the theta_u columns of the slot rows the binning kernel writes for the same
    projection, bit for bit (same fp32 expression)."""
    from tt_splat_b200 import binned, camera, ops
    from tt_splat_b200.model import pack_arrays
    sc = pkg.synthetic.config0(seed=3, G=1500, res=96)
    p = sc["params"]
    G = p["means3d"].shape[0]
    flat = pack_arrays(p).to(DEV)
    pj = ops.project(flat, G, 0, camera.pack_cameras([camera.Camera.from_dict(sc["cams"][0])], DEV), 96, 96)
    bp = ops.bin_pack(pj, G, 96, 96, 1, 128)
    tm = binned.TileMap(96, 96)
    idx = bp["idx"][0].long()
    valid = idx >= 0
    g = torch.where(valid, idx, torch.zeros_like(idx))
    th = binned.theta_u_gathered(pj["proj"][0, :, 2:5][g], pj["mu2d"][0][g], tm.origins, 4.0)
    rows = bp["slots"][0][..., 0:6].transpose(1, 2)
    vm = valid[:, None, :].expand_as(th)
    assert torch.equal(th[vm], rows[vm])
