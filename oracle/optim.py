"""Oracle: Adam, 3DGS-MCMC SGLD noise, relocation and the MCMC regulariser.

- Adam: ``torch.optim.Adam`` as constructed by ``spike/train.py:19`` (betas 0.9/0.999, eps 1e-8,
  per-group lr from ``spike/model.py:82-95``), single-tensor update order of torch:
  m.lerp_(g, 1-b1); v = v*b2 + (1-b2)*g*g; p += -(lr/bc1) * m / (sqrt(v)/sqrt(bc2) + eps).
  float32 like the reference.
- SGLD: ``add_sgld_noise`` (spike/mcmc.py:25-34) with the Gaussian draw injected.
- Relocation: ``relocate`` (spike/mcmc.py:41-71) with the multinomial targets (and the offset
  noise) injected, plus ``reset_adam_state`` (spike/mcmc.py:77-87).
- Regulariser gradient of ``reg_loss`` (spike/mcmc.py:18-22).
"""
import math

import numpy as np

from .geometry import quat_to_rotmat

F32 = np.float32
DEFAULT_LR = {"means": 5e-3, "scales": 5e-3, "quats": 1e-3, "opacity": 5e-2,
              "opacity_sh": 5e-2, "color": 1e-2, "wb": 1e-2, "depth": 1e-2}   # spike/train.py:9-12


def adam_update(p, g, m, v, step, lr, beta1=0.9, beta2=0.999, eps=1e-8):
    """One torch Adam step on float32 arrays (in place on p, m, v)."""
    w = F32(1.0 - beta1)
    m += w * (g - m)                                   # lerp_(grad, 1-beta1), weight < 0.5 branch
    v *= F32(beta2)
    v += (F32(1.0 - beta2) * g) * g                    # addcmul_(g, g, value=1-beta2)
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    step_size = lr / bc1
    denom = np.sqrt(v) / F32(math.sqrt(bc2)) + F32(eps)
    p += (F32(-step_size) * m) / denom                 # addcdiv_(m, denom, value=-step_size)
    return p


def sgld_noise(means, log_scales, quats, opacity_raw, eps, lr_means, noise_lr=5e5):
    """add_sgld_noise (spike/mcmc.py:25-34) with eps[G,3] given: returns the new means."""
    o = 1.0 / (1.0 + np.exp(-np.asarray(opacity_raw, np.float64)))
    s = np.exp(np.asarray(log_scales, np.float64))
    L = quat_to_rotmat(quats) * s[:, None, :]
    gate = 1.0 / (1.0 + np.exp(-100.0 * ((1.0 - o) - 0.995)))        # op_sigmoid (spike/mcmc.py:13-15)
    weight = gate * (noise_lr * lr_means)
    return np.asarray(means, np.float64) + np.einsum("gij,gj->gi", L, np.asarray(eps, np.float64)) * weight[:, None]


def quantile_threshold(o, frac):
    """torch.quantile(o, frac) (linear interpolation): the dead threshold of the 'lowest frac
    of opacities' relocation policy."""
    s = np.sort(np.asarray(o, np.float64))
    pos = frac * (s.size - 1)
    lo = int(math.floor(pos))
    hi = min(lo + 1, s.size - 1)
    return s[lo] + (pos - lo) * (s[hi] - s[lo])


def relocate(params, dead_thr, targets, offset_noise=None, offset=0.0):
    """relocate (spike/mcmc.py:41-71) on a dict of float32 arrays, with the sampled targets
    (one per dead slot, in ascending dead order) given.  Returns (n_moved, touched)."""
    o = 1.0 / (1.0 + np.exp(-params["opacity_raw"].astype(np.float32)))
    o = o.astype(np.float32)
    dead = np.nonzero(o < dead_thr)[0]
    alive = np.nonzero(o >= dead_thr)[0]
    if dead.size == 0 or alive.size == 0:
        return 0, np.zeros(0, np.int64)
    targets = np.asarray(targets, np.int64)
    assert targets.size == dead.size
    uniq, counts = np.unique(targets, return_counts=True)
    n_at = {int(t): int(c) + 1 for t, c in zip(uniq, counts)}
    new_o = {int(t): np.clip(o[int(t)] / F32(n_at[int(t)]), F32(1e-6), F32(1 - 1e-6)) for t in uniq}

    def logit(p):
        p = F32(p)
        return F32(np.log(p / (F32(1.0) - p)))

    for t in uniq:
        params["opacity_raw"][int(t)] = logit(new_o[int(t)])
    for i, (d, t) in enumerate(zip(dead.tolist(), targets.tolist())):
        add = 0.0 if offset_noise is None else F32(offset) * offset_noise[i]
        params["means3d"][d] = params["means3d"][t] + add
        params["log_scales"][d] = params["log_scales"][t]
        params["quats"][d] = params["quats"][t]
        params["color_dc"][d] = params["color_dc"][t]
        params["color_rest"][d] = params["color_rest"][t]
        params["opacity_raw"][d] = logit(new_o[t])
    touched = np.unique(np.concatenate([dead, uniq]))
    return dead.size, touched


def reg_loss_grads(opacity_raw, log_scales, lambda_o=0.01, lambda_s=0.01):
    """Gradient of reg_loss (spike/mcmc.py:18-22): lambda_o*mean(|o|) + lambda_s*mean(|s|)
    -> (d/dopacity_raw[G], d/dlog_scales[G,3])."""
    G = opacity_raw.shape[0]
    o = 1.0 / (1.0 + np.exp(-np.asarray(opacity_raw, np.float64)))
    s = np.exp(np.asarray(log_scales, np.float64))
    return lambda_o / G * o * (1.0 - o), lambda_s / (3.0 * G) * s
