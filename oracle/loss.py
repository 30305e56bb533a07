"""Oracle: the photometric loss (1-l)*L1 + l*(1-SSIM) and its manual gradient.

Restates ``spike/metrics.py:6-28`` (loss_fn with inputs clamped to [0,1] for SSIM only, window
shrunk for tiny images) on top of the reference's SSIM restatement ``tools/loss_manual.py``:
11-tap sigma-1.5 Gaussian window (``gauss_1d`` :28-31), valid separable filtering (``filt`` :44-49
and its transpose ``filt_T`` :52-55), ``ssim_fwd`` :58-75 and the manual gradient of
``loss_manual`` :78-105.  float64.  The clamp's gradient follows torch (passes at the bounds).
pytorch_msssim 1.0.0, the third-party package the reference calls, is not installed: its SSIM
is pinned through an independent restatement of its published algorithm (tests), not run.
"""
import numpy as np

C1 = 0.01 ** 2          # tools/loss_manual.py:21
C2 = 0.03 ** 2          # tools/loss_manual.py:22
SIGMA = 1.5             # tools/loss_manual.py:24


def ssim_window(H, W, win_size=11):
    """spike/metrics.py:15-19: win = min(win_size, H, W), made odd, at least 3."""
    win = min(win_size, H, W)
    if win % 2 == 0:
        win -= 1
    return max(win, 3)


def gauss_1d(win=11, sigma=SIGMA):
    """tools/loss_manual.py:28-31."""
    c = np.arange(win, dtype=np.float64) - win // 2
    g = np.exp(-(c ** 2) / (2 * sigma ** 2))
    return g / g.sum()


def filt(x, g):
    """Valid separable filter of x[C,H,W]: along H then along W (tools/loss_manual.py:44-49)."""
    win = g.size
    Ho, Wo = x.shape[1] - win + 1, x.shape[2] - win + 1
    t = sum(g[i] * x[:, i:i + Ho, :] for i in range(win))
    return sum(g[i] * t[:, :, i:i + Wo] for i in range(win))


def filt_T(m, g, H, W):
    """Transpose of ``filt`` (tools/loss_manual.py:52-55): [C,Ho,Wo] -> [C,H,W]."""
    win = g.size
    Ho, Wo = m.shape[1], m.shape[2]
    t = np.zeros((m.shape[0], Ho, W))
    for i in range(win):
        t[:, :, i:i + Wo] += g[i] * m
    out = np.zeros((m.shape[0], H, W))
    for i in range(win):
        out[:, i:i + Ho, :] += g[i] * t
    return out


def ssim_fwd(x, y, g):
    """tools/loss_manual.py:58-75: SSIM map S[C,Ho,Wo] and the intermediates."""
    fx, fy = filt(x, g), filt(y, g)
    fx2, fy2, fxy = filt(x * x, g), filt(y * y, g), filt(x * y, g)
    mux, muy = fx, fy
    mux2, muy2 = mux * mux, muy * muy
    sx, sy, sxy = fx2 - mux2, fy2 - muy2, fxy - mux * muy
    A1 = 2 * mux * muy + C1
    A2 = 2 * sxy + C2
    B1 = mux2 + muy2 + C1
    B2 = sx + sy + C2
    S = (A1 * A2) / (B1 * B2)
    return S, dict(mux=mux, muy=muy, A1=A1, A2=A2, B1=B1, B2=B2)


def loss_and_grad(pred, gt, lam=0.2, win_size=11):
    """loss_fn (spike/metrics.py:26-28) for pred/gt [H,W,3]: returns (loss, ssim, l1,
    dloss/dpred[H,W,3]) with the manual gradient of tools/loss_manual.py:78-105 and the [0,1]
    clamp of spike/metrics.py:6-7 applied to the SSIM inputs only."""
    pred = np.asarray(pred, np.float64)
    gt = np.asarray(gt, np.float64)
    H, W = pred.shape[:2]
    N = pred.size
    l1 = np.abs(pred - gt).mean()
    g_l1 = (1.0 - lam) * np.sign(pred - gt) / N
    x = np.transpose(np.clip(pred, 0.0, 1.0), (2, 0, 1))
    y = np.transpose(np.clip(gt, 0.0, 1.0), (2, 0, 1))
    g = gauss_1d(ssim_window(H, W, win_size))
    S, c = ssim_fwd(x, y, g)
    Ns = S.size
    ssim = S.mean()
    mux, muy, A1, A2, B1, B2 = c["mux"], c["muy"], c["A1"], c["A2"], c["B1"], c["B2"]
    D = B1 * B2
    dS_dfx2 = -S / B2
    dS_dfxy = 2 * A1 / D
    dS_dfx = (2.0 / D) * (muy * (A2 - A1) - S * mux * (B2 - B1))
    t1, t2, t3 = filt_T(dS_dfx, g, H, W), filt_T(dS_dfx2, g, H, W), filt_T(dS_dfxy, g, H, W)
    dmeanS_dx = (t1 + 2 * x * t2 + y * t3) / Ns
    mask = ((pred >= 0.0) & (pred <= 1.0)).astype(np.float64)
    g_ssim = lam * (-np.transpose(dmeanS_dx, (1, 2, 0))) * mask
    loss = (1.0 - lam) * l1 + lam * (1.0 - ssim)
    return loss, ssim, l1, g_l1 + g_ssim
