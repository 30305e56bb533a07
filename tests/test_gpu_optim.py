"""Fused Adam + SGLD and the relocation kernels vs torch's Adam, the reference MCMC (golden
fixtures with the random draws injected) and the oracle."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import optim as ooptim

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _flat(pkg, p):
    from tt_splat_b200.model import pack_arrays
    return pack_arrays(p).to(DEV)


def test_adam_matches_torch_optimizer(pkg):
    """Four steps of the fused kernel vs torch.optim.Adam (per-group lr) on the same grads."""
    from tt_splat_b200 import ops
    from tt_splat_b200.model import lr_vector, offsets
    from tt_splat_b200.train import DEFAULT_LR
    G = 777
    rng = np.random.default_rng(0)
    flat0 = torch.from_numpy(rng.standard_normal(59 * G + 1).astype(np.float32))
    lr = {**DEFAULT_LR, "means": 1.6e-4}
    off = offsets(G)
    params = {n: flat0[a:b].clone().requires_grad_(True) for n, (a, b) in off.items()}
    group_lr = dict(means3d=lr["means"], log_scales=lr["scales"], quats=lr["quats"], opacity_raw=lr["opacity"],
                    color_dc=lr["color"], color_rest=lr["color"] / 20.0, w_b_raw=lr["wb"])
    opt = torch.optim.Adam([{"params": [params[n]], "lr": group_lr[n]} for n in params])
    flat = flat0.clone().to(DEV)
    m, v = torch.zeros_like(flat), torch.zeros_like(flat)
    step = torch.zeros(1, dtype=torch.int32, device=DEV)
    lr7 = lr_vector(lr, DEV)
    for s in range(4):
        g = torch.from_numpy(rng.standard_normal(59 * G + 1).astype(np.float32) * 0.1)
        for n, (a, b) in off.items():
            params[n].grad = g[a:b].clone()
        opt.step()
        ops.step_begin(step)
        ops.adam_sgld(flat, g.to(DEV), m, v, G, 3, step, lr7)
    ref = torch.cat([params[n].detach() for n in off])
    err = (flat.cpu() - ref).abs().max().item()
    assert err <= 1e-6, err


def test_sgld_vs_reference(pkg):
    from tt_splat_b200 import ops
    z = golden("optim.npz")
    G = z["sgld_means3d"].shape[0]
    p = dict(means3d=z["sgld_means3d"], log_scales=z["sgld_log_scales"], quats=z["sgld_quats"],
             opacity_raw=z["sgld_opacity_raw"], color_dc=np.zeros((G, 3), np.float32), w_b_raw=-3.0)
    flat = _flat(pkg, p)
    step = torch.ones(1, dtype=torch.int32, device=DEV)
    ops.sgld(flat, G, step, 5e-3, 5e5, torch.from_numpy(z["sgld_eps"]).to(DEV))
    out = flat[:3 * G].view(G, 3).cpu().numpy()
    ref = z["sgld_out"]
    assert (np.abs(out - ref) <= 2e-5 * np.maximum(1.0, np.abs(ref))).all()


def test_relocate_vs_reference(pkg):
    from tt_splat_b200 import ops
    from tt_splat_b200.model import view
    z = golden("optim.npz")
    names = ("means3d", "log_scales", "quats", "color_dc", "color_rest", "opacity_raw")
    p = {k: z[f"reloc_in_{k}"] for k in names}
    p["w_b_raw"] = -3.0
    G = p["means3d"].shape[0]
    flat = _flat(pkg, p)
    m = torch.ones_like(flat)
    v = torch.ones_like(flat)
    step = torch.ones(1, dtype=torch.int32, device=DEV)
    out = ops.relocate(flat, m, v, G, step, 0.005, 0.0, 0.005,
                       torch.from_numpy(z["reloc_targets"].astype(np.int32)).to(DEV),
                       torch.from_numpy(z["reloc_noise"].astype(np.float32)).to(DEV))
    assert int(out["n_dead"]) == int(z["reloc_moved"])
    for k in names:
        got = view(flat, G, k).cpu().numpy()
        assert np.abs(got - z[f"reloc_out_{k}"]).max() < 1e-5, k
    touched = z["reloc_touched"]
    mm = view(m, G, "means3d").cpu().numpy()
    assert (mm[touched] == 0).all()
    untouched = np.setdiff1d(np.arange(G), touched)
    assert (mm[untouched] == 1).all()


def test_relocation_quantile_threshold_and_sampling(pkg):
    """dead_frac: the 1% lowest opacities are relocated (torch.quantile threshold); sampled
    targets are alive and the split preserves each target's summed opacity."""
    from tt_splat_b200 import ops
    from tt_splat_b200.model import view
    sc = pkg.synthetic.config0(seed=6, G=20000)
    p = sc["params"]
    flat = _flat(pkg, p)
    G = 20000
    o = 1 / (1 + np.exp(-p["opacity_raw"].astype(np.float64)))
    thr = ooptim.quantile_threshold(o.astype(np.float32), 0.01)
    n_expected = int((o.astype(np.float32) < np.float32(thr)).sum())
    m, v = torch.zeros_like(flat), torch.zeros_like(flat)
    step = torch.ones(1, dtype=torch.int32, device=DEV)
    out = ops.relocate(flat, m, v, G, step, 0.0, 0.01, 0.0, seed=7)
    n = int(out["n_dead"])
    assert n == n_expected == 200
    tg = out["targets"][:n].cpu().numpy()
    dead = np.argsort(o, kind="stable")[:n]
    assert not np.isin(tg, dead).any()
    o_new = 1 / (1 + np.exp(-view(flat, G, "opacity_raw").cpu().numpy().astype(np.float64)))
    for t in np.unique(tg)[:50]:
        c = int((tg == t).sum())
        assert abs(o_new[t] * (c + 1) - o[t]) < 1e-5
    # deterministic given (seed, step)
    flat2 = _flat(pkg, p)
    out2 = ops.relocate(flat2, torch.zeros_like(flat2), torch.zeros_like(flat2), G, step, 0.0, 0.01, 0.0, seed=7)
    assert torch.equal(out2["targets"][:n], out["targets"][:n]) and torch.equal(flat2, flat)


@pytest.mark.parametrize("injected", [False, True])
def test_sgld_relocate_equals_sgld_then_relocate(injected, pkg):
    """The one-launch SGLD + relocation of a relocating iteration gives the bits of tts_sgld
    followed by tts_relocate (Philox draws, and injected SGLD noise + relocation draws)."""
    from tt_splat_b200 import ops
    sc = pkg.synthetic.config2(seed=9, G=30000, H=64, W=96, n_views=1)
    G = 30000
    flat0 = _flat(pkg, sc["params"])
    rng = np.random.default_rng(3)
    m0 = torch.from_numpy(rng.standard_normal(flat0.numel()).astype(np.float32)).to(DEV)
    v0 = torch.from_numpy(rng.random(flat0.numel()).astype(np.float32)).to(DEV)
    step = torch.full((1,), 5, dtype=torch.int32, device=DEV)
    lr7 = torch.tensor([1.6e-4, 5e-3, 1e-3, 5e-2, 2.5e-3, 1.25e-4, 1e-3], dtype=torch.float64, device=DEV)
    eps = torch.from_numpy(rng.standard_normal((G, 3)).astype(np.float32)).to(DEV) if injected else None
    kw = dict(dead_thr=0.0, dead_frac=0.01, offset=0.3, seed=11)
    if injected:
        # injected targets drawn from the upper half of the opacities (alive: never a dead slot)
        o = sc["params"]["opacity_raw"].astype(np.float64)
        alive = np.argsort(o, kind="stable")[G // 2:]
        kw.update(targets_in=torch.from_numpy(rng.choice(alive, G).astype(np.int32)).to(DEV),
                  noise_in=torch.from_numpy(rng.standard_normal((G, 3)).astype(np.float32)).to(DEV))
    a, ma, va = flat0.clone(), m0.clone(), v0.clone()
    ops.sgld(a, G, step, 1.6e-4, 5e5, eps, seed=11)
    ra = ops.relocate(a, ma, va, G, step, kw["dead_thr"], kw["dead_frac"], kw["offset"], kw.get("targets_in"),
                      kw.get("noise_in"), seed=11)
    b, mb, vb = flat0.clone(), m0.clone(), v0.clone()
    rb = ops.sgld_relocate(b, mb, vb, G, step, lr7, 5e5, eps, **kw)
    n = int(ra["n_dead"])
    assert n == int(rb["n_dead"]) > 0
    assert torch.equal(ra["targets"][:n], rb["targets"][:n])
    assert torch.equal(a, b) and torch.equal(ma, mb) and torch.equal(va, vb)


@pytest.mark.parametrize("n_bucket", [3000, 10000])
def test_relocation_quantile_inside_one_bucket(n_bucket, pkg):
    """The 1% quantile lies among n_bucket opacities that share the select's first (11-bit) digit,
    spaced ~13 ulps apart: with 3000 members the last two digits are selected among them in
    shared memory, with 10000 (over the list capacity) by the grid-wide passes.  Either way the
    threshold falls between the 500th and 501st smallest opacity: the relocation is bit-identical
    to one given a threshold between those two values."""
    from tt_splat_b200 import ops
    G = 50000
    p = dict(pkg.synthetic.config0(seed=8, G=G)["params"])
    rng = np.random.default_rng(5)
    o = np.concatenate([0.0832 + 1e-7 * np.arange(n_bucket), rng.uniform(0.5, 0.95, G - n_bucket)])
    perm = rng.permutation(G)
    o = o[perm]
    p["opacity_raw"] = np.log(o / (1.0 - o)).astype(np.float32)
    flat0 = _flat(pkg, p)
    low = np.sort(o)[:501]
    assert low[-1] < 0.09375 and low[0] >= 0.078125          # one 11-bit bucket of the fp32 bits
    mid = float(0.5 * (low[499] + low[500]))
    step = torch.ones(1, dtype=torch.int32, device=DEV)
    outs = []
    for thr, frac in ((0.0, 0.01), (mid, 0.0)):
        flat = flat0.clone()
        m, v = torch.ones_like(flat), torch.ones_like(flat)
        r = ops.relocate(flat, m, v, G, step, thr, frac, 0.2, seed=21)
        outs.append((int(r["n_dead"]), r["targets"][:500].clone(), flat, m, v))
    (na, ta, fa, ma, va), (nb, tb, fb, mb, vb) = outs
    assert na == nb == 500
    assert torch.equal(ta, tb) and torch.equal(fa, fb) and torch.equal(ma, mb) and torch.equal(va, vb)
