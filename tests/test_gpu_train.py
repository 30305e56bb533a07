"""The graph-captured train step vs the oracle step, graph replay vs eager, and training."""
import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import pipeline

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _setup(pkg, seed=0, G=3000, res=64, views=2, deg=3):
    sc = pkg.synthetic.config2(seed=seed, G=G, H=res, W=res + 32, n_views=views)
    return sc


def test_one_step_vs_oracle(pkg):
    """Loss, gradient and the Adam update of one device step vs the oracle step."""
    from tt_splat_b200 import camera, model, train
    sc = _setup(pkg)
    p = sc["params"]
    m = model.GaussianModel.from_arrays(p, device=DEV)
    st = train.TrainStep(m, [camera.Camera.from_dict(c) for c in sc["cams"]],
                         [torch.from_numpy(t) for t in sc["targets"]], sh_degree=3, lr={"means": 1.6e-4},
                         lambda_o=0.01, lambda_s=0.01, use_graph=False)
    st.step()
    total, losses, grads = pipeline.loss_and_grads(p, sc["cams"], sc["targets"], 3, lambda_o=0.01, lambda_s=0.01)
    assert abs(st.mean_loss_value() - total) < 1e-4 * total
    G = p["means3d"].shape[0]
    for n in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest"):
        assert rel_l2(model.view(st.grads, G, n).cpu().numpy(), grads[n]) < 1e-3, n
    # the Adam update: the oracle's torch-order Adam applied to the device gradient (a first Adam
    # step is ~lr * sign(g), so comparing updates of two gradients that differ in the last bits
    # would test the sign of near-zero components, not the update)
    dev_g = {n: model.view(st.grads, G, n).cpu().numpy() for n in ("means3d", "log_scales", "quats", "opacity_raw",
                                                                     "color_dc", "color_rest")}
    dev_g["w_b_raw"] = np.float32(model.view(st.grads, G, "w_b_raw").item())
    ref = pipeline.copy_params(p)
    pipeline.adam_step(ref, dev_g, {}, 1, {**train.DEFAULT_LR, "means": 1.6e-4}, 3)
    for n in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest"):
        d = np.abs(model.view(m.flat.data, G, n).cpu().numpy() - ref[n]).max()
        assert d <= 1e-6, (n, d)


@pytest.mark.parametrize("arm", ["B", "RV"])
def test_one_step_arms_vs_oracle(arm, pkg):
    """Arms B and RV through the train step: loss and gradients (the depth pair under B) vs the
    oracle, and the depth group's Adam update vs torch's formula."""
    from oracle import optim as ooptim
    from tt_splat_b200 import camera, model, train
    sc = _setup(pkg, seed=4)
    p = sc["params"]
    m = model.GaussianModel.from_arrays(p, device=DEV)
    bt = (1.3, 3.9)
    with torch.no_grad():
        m.depth_beta.fill_(bt[0])
        m.depth_tau.fill_(bt[1])
    st = train.TrainStep(m, [camera.Camera.from_dict(c) for c in sc["cams"]],
                         [torch.from_numpy(t) for t in sc["targets"]], sh_degree=3, use_graph=False, arm=arm)
    st.step()
    total, _, grads = pipeline.loss_and_grads(p, sc["cams"], sc["targets"], 3, depth_bt=bt if arm == "B" else None,
                                              arm=arm)
    assert abs(st.mean_loss_value() - total) < 1e-4 * total
    G = p["means3d"].shape[0]
    for n in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest"):
        assert rel_l2(model.view(st.grads, G, n).cpu().numpy(), grads[n]) < 1e-3, n
    if arm == "RV":
        assert float(model.view(st.grads, G, "w_b_raw")) == 0.0
        assert float(model.view(m.flat.data, G, "w_b_raw")) == float(p["w_b_raw"])   # no gradient, no update
        return
    g = st.g_dbt.cpu().numpy()
    ref_g = np.array([grads["depth_beta"], grads["depth_tau"]])
    assert np.abs(g - ref_g).max() < 1e-3 * np.abs(ref_g).max()
    pd = np.array(bt, np.float32)
    ooptim.adam_update(pd, g.astype(np.float32), np.zeros(2, np.float32), np.zeros(2, np.float32), 1,
                       train.DEFAULT_LR["depth"])
    assert float(m.depth_beta) == pytest.approx(float(pd[0]), abs=1e-6)
    assert float(m.depth_tau) == pytest.approx(float(pd[1]), abs=1e-6)
    assert abs(float(m.depth_beta) - bt[0]) > 1e-3            # the depth pair trained


def test_graph_replay_equals_eager(pkg):
    from tt_splat_b200 import camera, model, train
    sc = _setup(pkg, seed=1)
    cams = [camera.Camera.from_dict(c) for c in sc["cams"]]
    tg = [torch.from_numpy(t) for t in sc["targets"]]
    m1 = model.GaussianModel.from_arrays(sc["params"], device=DEV)
    m2 = model.GaussianModel.from_arrays(sc["params"], device=DEV)
    kw = dict(sh_degree=3, noise_lr=5e5, relocate_every=2, dead_thr=0.005, offset=0.005, lambda_o=0.01, lambda_s=0.01,
              seed=3)
    a = train.TrainStep(m1, cams, tg, use_graph=True, **kw)
    b = train.TrainStep(m2, cams, tg, use_graph=False, **kw)
    for _ in range(5):
        la, lb = a.step(), b.step()
        assert torch.equal(la, lb)
    assert torch.equal(m1.flat, m2.flat)
    assert len(a.graphs) == 2


def test_training_reduces_loss(pkg):
    from tt_splat_b200 import camera, mcmc, model
    sc = _setup(pkg, seed=2, G=2000, res=48, views=3)
    target_model = model.GaussianModel.from_arrays(sc["params"], device=DEV)
    cams = [camera.Camera.from_dict(c) for c in sc["cams"]]
    from tt_splat_b200 import render
    with torch.no_grad():
        gts = [render.render(target_model, c, sh_degree=3).detach() for c in cams]
    fresh = pkg.synthetic.config2(seed=9, G=2000, H=48, W=80, n_views=1)["params"]
    m = model.GaussianModel.from_arrays(fresh, device=DEV)
    hist, moved = mcmc.train_mcmc(m, cams, gts, iters=120, relocate_every=40, noise_lr=50.0, sh_degree=3)
    assert hist[-1] < 0.7 * hist[0], (hist[0], hist[-1])
    assert moved >= 0


def test_uint8_targets_equal_float_targets(pkg):
    """A train step given 8-bit targets (expanded on the device to x / 255, correctly rounded)
    takes bit-identical steps to one given the float targets numpy computes from them."""
    from tt_splat_b200 import camera, model, ops, train
    sc = pkg.synthetic.config2(seed=6, G=2000, H=48, W=64, n_views=2)
    u8 = torch.from_numpy(np.stack(sc["targets_u8"])).to(DEV)
    f = ops.unit_from_u8(u8)
    assert torch.equal(f.cpu(), torch.from_numpy(np.stack(sc["targets"])))
    cams = [camera.Camera.from_dict(c) for c in sc["cams"]]
    kw = dict(sh_degree=3, noise_lr=5e5, relocate_every=2, dead_frac=0.01, offset=0.005, seed=2)
    m1 = model.GaussianModel.from_arrays(sc["params"], device=DEV)
    m2 = model.GaussianModel.from_arrays(sc["params"], device=DEV)
    a = train.TrainStep(m1, cams, sc["targets_u8"], **kw)
    b = train.TrainStep(m2, cams, sc["targets"], **kw)
    assert a.targets_u8 is not None and b.targets_u8 is None
    for _ in range(4):
        assert torch.equal(a.step(), b.step())
    assert torch.equal(m1.flat, m2.flat)
