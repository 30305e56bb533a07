"""3DGS-MCMC on the device (mirrors spike/mcmc.py:1-114).

``train_mcmc`` runs the graph-captured ``TrainStep`` with the fused Adam + SGLD kernel and the
relocation kernels; ``add_sgld_noise`` and ``relocate`` are the standalone reference entry
points on a model's flat buffer.
"""
import torch

from . import ops
from .model import GaussianModel, view
from .train import DEFAULT_LR, TrainStep


def op_sigmoid(x, k=100.0, x0=0.995):
    """spike/mcmc.py:13-15."""
    return torch.sigmoid(k * (x - x0))


def reg_loss(model, lambda_o=0.01, lambda_s=0.01):
    """spike/mcmc.py:18-22."""
    o = torch.sigmoid(model.opacity_raw)
    s = torch.exp(model.log_scales)
    return lambda_o * o.abs().mean() + lambda_s * s.abs().mean()


def _check(model):
    if not isinstance(model, GaussianModel):
        raise TypeError("expects a tt_splat_b200.model.GaussianModel (flat device buffer)")


@torch.no_grad()
def add_sgld_noise(model, lr, noise_lr=5e5, eps=None, seed=0, step=0):
    """spike/mcmc.py:25-34 on the device; ``eps[G,3]`` injects the Gaussian draw (else Philox)."""
    _check(model)
    st = torch.full((1,), int(step), dtype=torch.int32, device=model.flat.device)
    ops.sgld(model.flat.data, model.G, st, lr, noise_lr, None if eps is None else eps.float().contiguous(), seed)


@torch.no_grad()
def relocate(model, dead_thr=0.005, offset=0.0, targets=None, noise=None, dead_frac=0.0, seed=0, step=0,
             moments=None):
    """spike/mcmc.py:41-71 on the device; returns (n_moved, touched indices).  ``targets`` /
    ``noise`` inject the multinomial draw and the offset noise; ``moments = (m, v)`` are zeroed at
    the touched gaussians (reset_adam_state, spike/mcmc.py:77-87)."""
    _check(model)
    dev = model.flat.device
    G = model.G
    m, v = moments if moments is not None else (torch.zeros_like(model.flat), torch.zeros_like(model.flat))
    st = torch.full((1,), int(step), dtype=torch.int32, device=dev)
    tin = None if targets is None else torch.as_tensor(targets, dtype=torch.int32, device=dev).contiguous()
    nin = None if noise is None else torch.as_tensor(noise, dtype=torch.float32, device=dev).contiguous()
    o_before = torch.sigmoid(view(model.flat.data, G, "opacity_raw")).clone()
    out = ops.relocate(model.flat.data, m, v, G, st, dead_thr, dead_frac, offset, tin, nin, seed)
    n = int(out["n_dead"].item())
    if n == 0:
        return 0, torch.empty(0, dtype=torch.long, device=dev)
    thr = dead_thr if dead_frac <= 0 else None
    dead = torch.where(o_before < thr)[0] if thr is not None else None
    tg = out["targets"][:n].long()
    touched = torch.unique(torch.cat([dead, tg])) if dead is not None else torch.unique(tg)
    return n, touched


def reset_adam_state(step, idx):
    """spike/mcmc.py:77-87 for a TrainStep's moments."""
    if idx.numel() == 0:
        return
    G = step.G
    for name in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest"):
        view(step.m, G, name)[idx] = 0
        view(step.v, G, name)[idx] = 0


def train_mcmc(model, cameras, gt_images, arm="A", iters=600, lr=None, relocate_every=100, dead_thr=0.005,
               offset=0.005, lambda_o=0.01, lambda_s=0.01, noise_lr=5e5, k=4.0, blur_eps=0.3, near=0.2, log_every=0,
               sh_degree=0, dead_frac=0.0, K=128, R=1, seed=0):
    """spike/mcmc.py:90-114 on the B200 path -> (loss history, total relocations)."""
    st = TrainStep(model, cameras, gt_images, sh_degree=sh_degree, lr={**DEFAULT_LR, **(lr or {})}, K=K, R=R, k=k,
                   blur=blur_eps, near=near, noise_lr=noise_lr, relocate_every=relocate_every, dead_thr=dead_thr,
                   dead_frac=dead_frac, offset=offset, lambda_o=lambda_o, lambda_s=lambda_s, seed=seed, arm=arm)
    hist = []
    for it in range(iters):
        st.step()
        hist.append(st.mean_loss_value() if log_every else st.loss_mean.clone())
        if log_every and (it % log_every == 0 or it == iters - 1):
            print(f"    iter {it:4d}  loss {hist[-1]:.5f}  relocations {int(st.n_moved.item())}")
    st.check_status()
    if hist and torch.is_tensor(hist[0]):
        hist = (torch.cat(hist) / st.V).cpu().tolist()
    return hist, int(st.n_moved.item())
