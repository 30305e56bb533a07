"""The headline workload (benchmark config 2) at its own size against the oracle.

G = 100,000 gaussians, SH degree 3, the 8-view ring batch at 1264x832, K = 128, R = 1,
0.8 L1 + 0.2 (1 - SSIM), the MCMC regulariser (0.01, 0.01) and Adam with lr 1.6e-4 on the
means: exactly the scene and settings ``bench.py`` times.  One eager device step is compared
with the oracle step on the same inputs (spike/mcmc.py:90-114 order: loss, gradient, Adam):

* the mean photometric loss to 1e-4 relative;
* every parameter block's gradient to 1e-3 relative L2 (north_star's fp32 gradient bound);
* the Adam update: the device's updated parameters equal the oracle's torch-order Adam applied
  to the device gradient (so the update arithmetic is checked apart from the gradient).

SGLD noise and relocation are random draws (Philox on the device); at G = 100k they are checked
with the oracle's draws injected, as the reference's own MCMC tests inject theirs.
"""
import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import optim as ooptim
from oracle import pipeline

pytestmark = pytest.mark.gpu
DEV = "cuda"
NAMES = ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest")
LR = {"means": 1.6e-4}


@pytest.fixture(scope="module")
def headline(pkg):
    """The config-2 scene and the oracle's loss and gradient for it (the 8 views' forward, loss
    and backward on spawned worker processes, summed in view order)."""
    from oracle.step import CpuStep
    sc = pkg.synthetic.config2()
    with CpuStep(sc) as cs:
        loss, grads = cs.loss_and_grads(lambda_o=0.01, lambda_s=0.01)
    return sc, loss, grads


def test_headline_step_vs_oracle(headline):
    from tt_splat_b200 import camera, model, train
    sc, loss, grads = headline
    p = sc["params"]
    G = p["means3d"].shape[0]
    assert G == 100000 and len(sc["cams"]) == 8 and sc["cams"][0]["W"] == 1264 and sc["cams"][0]["H"] == 832
    m = model.GaussianModel.from_arrays(p, device=DEV)
    st = train.TrainStep(m, [camera.Camera.from_dict(c) for c in sc["cams"]],
                         [torch.from_numpy(t) for t in sc["targets"]], sh_degree=3, lr=LR, K=128, R=1,
                         lambda_o=0.01, lambda_s=0.01, use_graph=False)
    st.step()
    st.check_status()
    dev_loss = float(st.loss_mean.item()) / st.V          # the photometric part (mean over views)
    assert abs(dev_loss - loss) < 1e-4 * loss, (dev_loss, loss)
    for n in NAMES:
        err = rel_l2(model.view(st.grads, G, n).cpu().numpy(), grads[n])
        assert err < 1e-3, (n, err)
    gwb = float(model.view(st.grads, G, "w_b_raw"))
    assert abs(gwb - grads["w_b_raw"]) < 1e-3 * abs(grads["w_b_raw"]), (gwb, grads["w_b_raw"])
    # Adam: the oracle's torch-order update applied to the device gradient
    dev_g = {n: model.view(st.grads, G, n).cpu().numpy() for n in NAMES}
    dev_g["w_b_raw"] = np.float32(gwb)
    ref = pipeline.copy_params(p)
    pipeline.adam_step(ref, dev_g, {}, 1, {**train.DEFAULT_LR, **LR}, 3)
    for n in NAMES:
        d = np.abs(model.view(m.flat.data, G, n).cpu().numpy() - ref[n]).max()
        assert d <= 1e-6, (n, d)
    assert abs(float(model.view(m.flat.data, G, "w_b_raw")) - float(ref["w_b_raw"])) <= 1e-6


def test_headline_sgld_and_relocation_with_injected_draws(pkg):
    """add_sgld_noise (spike/mcmc.py:25-34) and relocate + reset_adam_state (:41-87) over the
    100k gaussians of the headline scene, with the oracle's Gaussian draw, multinomial targets
    and offset noise injected: the 1% lowest opacities move (threshold placed between the
    1000th and 1001st opacity so that no gaussian sits on it)."""
    from tt_splat_b200 import ops
    from tt_splat_b200.model import pack_arrays, view
    p = pkg.synthetic.config2()["params"]
    G = p["means3d"].shape[0]
    rng = np.random.default_rng(17)
    flat = pack_arrays(p).to(DEV)
    step = torch.ones(1, dtype=torch.int32, device=DEV)
    eps = rng.standard_normal((G, 3)).astype(np.float32)
    ops.sgld(flat, G, step, LR["means"], 5e5, torch.from_numpy(eps).to(DEV))
    ref_means = ooptim.sgld_noise(p["means3d"], p["log_scales"], p["quats"], p["opacity_raw"], eps, LR["means"])
    got = view(flat, G, "means3d").cpu().numpy()
    assert (np.abs(got - ref_means) <= 2e-5 * np.maximum(1.0, np.abs(ref_means))).all()

    q = {k: np.array(p[k], np.float32, copy=True) for k in NAMES}
    q["means3d"] = got.copy()
    o = (1.0 / (1.0 + np.exp(-q["opacity_raw"].astype(np.float32)))).astype(np.float32)
    so = np.sort(o)
    # about 1% dead, at a gap of several ulps so that a last-bit difference between the device's
    # and numpy's sigmoid cannot move a gaussian across the threshold
    n_dead = next(n for n in range(G // 100, G // 100 + 200) if so[n] - so[n - 1] > 8 * np.spacing(so[n]))
    thr = float(so[n_dead - 1]) + 0.5 * float(so[n_dead] - so[n_dead - 1])
    dead = np.nonzero(o < thr)[0]
    alive = np.nonzero(o >= thr)[0]
    assert dead.size == n_dead
    tg = alive[rng.choice(alive.size, n_dead, p=o[alive].astype(np.float64) / o[alive].astype(np.float64).sum())]
    noise = rng.standard_normal((n_dead, 3)).astype(np.float32)
    mom_m, mom_v = torch.ones_like(flat), torch.ones_like(flat)
    out = ops.relocate(flat, mom_m, mom_v, G, step, thr, 0.0, 0.005, torch.from_numpy(tg.astype(np.int32)).to(DEV),
                       torch.from_numpy(noise).to(DEV))
    assert int(out["n_dead"]) == n_dead
    n_ref, touched = ooptim.relocate(q, np.float32(thr), tg, noise, 0.005)
    assert n_ref == n_dead
    for k in NAMES:
        d = np.abs(view(flat, G, k).cpu().numpy() - q[k]).max()
        assert d < 1e-5, (k, d)
    for k in NAMES:
        mm = view(mom_m, G, k).cpu().numpy().reshape(G, -1)
        vv = view(mom_v, G, k).cpu().numpy().reshape(G, -1)
        assert (mm[touched] == 0).all() and (vv[touched] == 0).all(), k
        untouched = np.setdiff1d(np.arange(G), touched)
        assert (mm[untouched] == 1).all() and (vv[untouched] == 1).all(), k
