"""Functional wrappers over the C ABI: allocate outputs with torch, call on the current stream.

Shapes follow ``include/ttsplat_b200.h``.  Every function validates that its tensors are CUDA
and contiguous and raises otherwise (no CPU fallback).
"""
import numpy as np
import torch

from ._lib import call, lib, ptr, stream

SLOT_FLOATS = 12
SLOT_GRAD_FLOATS = 10
SLOT_BF16 = 16          # compact bf16 slot row: theta hi[6], theta lo[6], color_o[3], o_col
PROJ_FLOATS = 12


def _dev(*ts):
    """CUDA, contiguous, and on the current device (the library launches on the current device's
    current stream)."""
    cur = None
    for t in ts:
        if t is not None:
            if not t.is_cuda:
                raise RuntimeError("tt-splat B200 ops need CUDA tensors (no CPU fallback)")
            if not t.is_contiguous():
                raise ValueError("tensors must be contiguous")
            if cur is None:
                cur = torch.cuda.current_device()
            if t.device.index != cur:
                raise ValueError(f"tensor on {t.device} but the current device is cuda:{cur}: "
                                 "call under torch.cuda.device(...) of the tensors' device")


def tiles(H, W):
    if H % 16 or W % 16:
        raise AssertionError("H and W must be multiples of 16 (TileMap, tools/m4_train_binned.py:62)")
    return W // 16, H // 16, (W // 16) * (H // 16)


class Workspace:
    """A grow-only device scratch buffer."""

    def __init__(self, device):
        self.device = device
        self.buf = torch.empty(0, dtype=torch.uint8, device=device)

    def get(self, nbytes):
        if self.buf.numel() < nbytes:
            self.buf = torch.empty(int(nbytes), dtype=torch.uint8, device=self.device)
        return self.buf


def project(flat, G, sh_degree, cams, H, W, blur=0.3, near=0.2, out=None, depth_bt=None):
    """Geometry + SH + activations for V = cams.shape[0] views (also counts home cells);
    ``depth_bt`` (device [depth_beta, depth_tau]) selects arm B's depth-weighted opacity."""
    _dev(flat, cams, depth_bt)
    V = cams.shape[0]
    _, _, T = tiles(H, W)
    dev = flat.device
    if out is None:
        out = dict(proj=torch.empty(V, G, PROJ_FLOATS, device=dev), mu2d=torch.empty(V, G, 2, device=dev),
                   keep=torch.empty(V, G, dtype=torch.uint8, device=dev),
                   cell_count=torch.empty(V, T, dtype=torch.int32, device=dev),
                   cell_rank=torch.empty(V, G, 2, dtype=torch.int32, device=dev))
    call("tts_project", ptr(flat), G, sh_degree, ptr(cams), V, H, W, float(blur), float(near), ptr(out["proj"]),
         ptr(out["mu2d"]), ptr(out["keep"]), ptr(out["cell_count"]), ptr(out["cell_rank"]), ptr(depth_bt), stream())
    return out


def bin_from_mu2d(mu2d, keep, H, W, R, K, ws=None, with_inv=True):
    """assign_bins on given mu2d[V,G,2] / keep[V,G] (uint8 or bool)."""
    if mu2d.dim() == 2:
        mu2d, keep = mu2d[None], keep[None]
    keep = keep.to(torch.uint8).contiguous()
    mu2d = mu2d.float().contiguous()
    _dev(mu2d, keep)
    V, G = mu2d.shape[0], mu2d.shape[1]
    _, _, T = tiles(H, W)
    dev = mu2d.device
    S = (2 * R + 1) ** 2
    idx = torch.empty(V, T, K, dtype=torch.int32, device=dev)
    count = torch.empty(V, T, dtype=torch.int32, device=dev)
    cand = torch.empty(V, T, dtype=torch.int32, device=dev)
    inv = torch.empty(V, G, S, dtype=torch.int32, device=dev) if with_inv else None
    nbytes = lib().tts_bin_workspace_bytes(G, V, H, W)
    ws = ws or Workspace(dev)
    buf = ws.get(nbytes)
    call("tts_bin_from_mu2d", ptr(mu2d), ptr(keep), G, V, H, W, R, K, ptr(idx), ptr(count), ptr(cand), ptr(inv),
         ptr(buf), nbytes, stream())
    return idx, count, cand, inv


def bin_pack(pj, G, H, W, R, K, k=4.0, ws=None, out=None, with_inv=True, bf16=False):
    """Binning + slot-row pack on the output of ``project`` (``with_inv=False``: no inverse table,
    for forward-only rendering; ``bf16``: compact bf16 slot rows for the bf16 forward)."""
    V = pj["proj"].shape[0]
    _, _, T = tiles(H, W)
    dev = pj["proj"].device
    S = (2 * R + 1) ** 2
    if out is None:
        slots = (torch.empty(V, T, K, SLOT_BF16, dtype=torch.bfloat16, device=dev) if bf16
                 else torch.empty(V, T, K, SLOT_FLOATS, device=dev))
        out = dict(idx=torch.empty(V, T, K, dtype=torch.int32, device=dev),
                   count=torch.empty(V, T, dtype=torch.int32, device=dev),
                   cand=torch.empty(V, T, dtype=torch.int32, device=dev),
                   inv=torch.empty(V, G, S, dtype=torch.int32, device=dev) if with_inv else None,
                   slots=slots)
    fmt = 1 if out["slots"].dtype == torch.bfloat16 else 0
    nbytes = lib().tts_bin_workspace_bytes(G, V, H, W)
    ws = ws or Workspace(dev)
    buf = ws.get(nbytes)
    call("tts_bin_pack", ptr(pj["mu2d"]), ptr(pj["keep"]), ptr(pj["proj"]), ptr(pj["cell_count"]), ptr(pj["cell_rank"]),
         G, V, H, W, R, K, float(k), ptr(out["idx"]), ptr(out["count"]), ptr(out["cand"]), ptr(out["inv"]),
         ptr(out["slots"]), fmt, ptr(buf), nbytes, stream())
    return out


def pack_cached(pj, G, H, W, R, K, idx_in, k=4.0, ws=None):
    """Slot rows of the current projection for cached tables ``idx_in`` [V,T,K] (int32, -1 =
    invalid, valid slots first), with the count per tile and the inverse table."""
    _dev(pj["proj"], idx_in)
    V = pj["proj"].shape[0]
    _, _, T = tiles(H, W)
    if idx_in.dtype != torch.int32 or tuple(idx_in.shape) != (V, T, K):
        raise ValueError(f"cached idx must be int32 [{V}, {T}, {K}]")
    dev = pj["proj"].device
    S = (2 * R + 1) ** 2
    out = dict(idx=torch.empty_like(idx_in), count=torch.empty(V, T, dtype=torch.int32, device=dev),
               inv=torch.empty(V, G, S, dtype=torch.int32, device=dev), slots=torch.zeros(V, T, K, SLOT_FLOATS, device=dev))
    nbytes = lib().tts_pack_cached_workspace_bytes(G, V)
    ws = ws or Workspace(dev)
    buf = ws.get(nbytes)
    call("tts_pack_cached", ptr(pj["proj"]), G, V, H, W, R, K, float(k), ptr(idx_in), ptr(out["idx"]), ptr(out["count"]),
         ptr(out["inv"]), ptr(out["slots"]), ptr(buf), nbytes, stream())
    return out


def render_fwd(slots, count, H, W, w_b, c_b, bf16=False, out=None, w_b_is_raw=True):
    """Per-tile forward; ``w_b`` is a 1-element device tensor: the model's w_b_raw (softplus
    applied on the device) or, with ``w_b_is_raw=False``, the activated background weight."""
    _dev(slots, count, w_b, c_b)
    V, T, K = slots.shape[0], slots.shape[1], slots.shape[2]
    dev = slots.device
    if out is None:
        out = dict(img=torch.empty(V, H, W, 3, device=dev), den=torch.empty(V, H, W, device=dev))
    call("tts_render_fwd", ptr(slots), int(bool(bf16)), ptr(count), V, H, W, K, ptr(w_b), int(bool(w_b_is_raw)), ptr(c_b),
         ptr(out["img"]), ptr(out["den"]), stream())
    return out


def render_bwd(slots, count, H, W, c_b, img, den, gimg, out=None):
    _dev(slots, count, c_b, img, den, gimg)
    V, T, K = slots.shape[0], slots.shape[1], slots.shape[2]
    dev = slots.device
    if out is None:
        out = dict(slot_grads=torch.empty(V, T, K, SLOT_GRAD_FLOATS, device=dev), gwb=torch.empty(V, T, device=dev))
    call("tts_render_bwd", ptr(slots), ptr(count), V, H, W, K, ptr(c_b), ptr(img), ptr(den), ptr(gimg),
         ptr(out["slot_grads"]), ptr(out["gwb"]), stream())
    return out


def render_fwd_rv(slots, count, H, W, c_b, out=None):
    """Arm RV per-tile forward (fp32 slot rows) -> img, den and aux = (Cavg, R) per pixel."""
    _dev(slots, count, c_b)
    V, T, K = slots.shape[0], slots.shape[1], slots.shape[2]
    dev = slots.device
    if out is None:
        out = dict(img=torch.empty(V, H, W, 3, device=dev), den=torch.empty(V, H, W, device=dev),
                   aux=torch.empty(V, H, W, 4, device=dev))
    call("tts_render_fwd_rv", ptr(slots), ptr(count), V, H, W, K, ptr(c_b), ptr(out["img"]), ptr(out["den"]),
         ptr(out["aux"]), stream())
    return out


def render_bwd_rv(slots, count, H, W, c_b, den, aux, gimg, out=None):
    _dev(slots, count, c_b, den, aux, gimg)
    V, T, K = slots.shape[0], slots.shape[1], slots.shape[2]
    dev = slots.device
    if out is None:
        out = dict(slot_grads=torch.empty(V, T, K, SLOT_GRAD_FLOATS, device=dev), gwb=torch.empty(V, T, device=dev))
    call("tts_render_bwd_rv", ptr(slots), ptr(count), V, H, W, K, ptr(c_b), ptr(den), ptr(aux), ptr(gimg),
         ptr(out["slot_grads"]), ptr(out["gwb"]), stream())
    return out


def loss_l1_ssim(img, target, lam=0.2, grad_scale=1.0, ws=None, out=None):
    """(1-lam) L1 + lam (1 - SSIM) of img [V,H,W,3] against target (both fp32)
    -> dict(gimg = grad_scale * dloss/dimg, loss[V])."""
    _dev(img, target)
    if img.dim() == 3:
        img, target = img[None], target[None]
    V, H, W = img.shape[0], img.shape[1], img.shape[2]
    dev = img.device
    if out is None:
        out = dict(gimg=torch.empty_like(img), loss=torch.empty(V, device=dev))
    nbytes = lib().tts_loss_workspace_bytes(V, H, W)
    ws = ws or Workspace(dev)
    buf = ws.get(nbytes)
    call("tts_loss_l1_ssim", ptr(img), ptr(target), V, H, W, float(lam), float(grad_scale), ptr(out["gimg"]),
         ptr(out["loss"]), ptr(out.get("loss_sum")), ptr(buf), nbytes, stream())
    return out


def backward_params(flat, G, sh_degree, cams, H, W, R, K, inv, slot_grads, gwb, k=4.0, blur=0.3, near=0.2,
                    lambda_o=0.0, lambda_s=0.0, out=None, ws=None, proj=None, depth_bt=None, g_depth_bt=None):
    """Parameter gradient from the per-slot gradients; ``proj`` is the projection of the same
    parameters and cameras (recomputed when not given).  Arm B: ``depth_bt`` as given to
    ``project``; d/d(depth_beta, depth_tau) goes to ``g_depth_bt`` (allocated when not given)."""
    _dev(flat, cams, inv, slot_grads, gwb, depth_bt)
    V = cams.shape[0]
    if proj is None:
        proj = project(flat, G, sh_degree, cams, H, W, blur, near, depth_bt=depth_bt)["proj"]
    if depth_bt is not None and g_depth_bt is None:
        g_depth_bt = torch.empty(2, device=flat.device)
    grads = out if out is not None else torch.empty_like(flat)
    nbytes = lib().tts_backward_workspace_bytes(G, V)
    ws = ws or Workspace(flat.device)
    buf = ws.get(nbytes)
    call("tts_backward_params", ptr(flat), G, sh_degree, ptr(cams), V, H, W, R, K, float(k), float(blur), float(near),
         ptr(proj), ptr(inv), ptr(slot_grads), ptr(gwb), float(lambda_o), float(lambda_s), ptr(grads), ptr(depth_bt),
         ptr(g_depth_bt), ptr(buf), nbytes, stream())
    return grads if depth_bt is None else (grads, g_depth_bt)


def sgld(flat, G, step, lr_means, noise_lr, eps_noise=None, seed=0):
    _dev(flat, step, eps_noise)
    call("tts_sgld", ptr(flat), G, float(lr_means), float(noise_lr), ptr(eps_noise), ptr(step),
         int(seed) & (2 ** 64 - 1), stream())


def adam_vec(p, g, m, v, step, lr, beta1=0.9, beta2=0.999, eps=1e-8):
    """Adam on a short device vector with one learning rate (the arm-B depth group)."""
    _dev(p, g, m, v, step)
    call("tts_adam_vec", ptr(p), ptr(g), ptr(m), ptr(v), p.numel(), ptr(step), float(lr), float(beta1), float(beta2),
         float(eps), stream())


def step_begin(step):
    call("tts_step_begin", ptr(step), stream())


def adam_sgld(flat, grads, m, v, G, sh_degree, step, lr7, betas=(0.9, 0.999), eps=1e-8, noise_lr=0.0,
              eps_noise=None, seed=0):
    _dev(flat, grads, m, v, step, lr7)
    call("tts_adam_sgld", ptr(flat), ptr(grads), ptr(m), ptr(v), G, sh_degree, ptr(step), ptr(lr7), float(betas[0]),
         float(betas[1]), float(eps), float(noise_lr), ptr(eps_noise), int(seed) & (2 ** 64 - 1), stream())


def relocate(flat, m, v, G, step, dead_thr=0.005, dead_frac=0.0, offset=0.0, targets_in=None, noise_in=None, seed=0,
             ws=None, out=None):
    _dev(flat, m, v, step)
    dev = flat.device
    if out is None:
        out = dict(n_dead=torch.zeros(1, dtype=torch.int32, device=dev),
                   targets=torch.empty(G, dtype=torch.int32, device=dev))
    nbytes = lib().tts_relocate_workspace_bytes(G)
    ws = ws or Workspace(dev)
    buf = ws.get(nbytes)
    call("tts_relocate", ptr(flat), ptr(m), ptr(v), G, float(dead_thr), float(dead_frac), float(offset), ptr(targets_in),
         ptr(noise_in), ptr(step), int(seed) & (2 ** 64 - 1), ptr(out["n_dead"]), ptr(out["targets"]), ptr(buf), nbytes,
         stream())
    return out


def sgld_relocate(flat, m, v, G, step, lr7, noise_lr, eps_noise=None, dead_thr=0.005, dead_frac=0.0, offset=0.0,
                  targets_in=None, noise_in=None, seed=0, ws=None, out=None):
    """sgld(...) then relocate(...) in one launch (the MCMC order of a relocating iteration);
    ``lr7`` is the device learning-rate table (means first)."""
    _dev(flat, m, v, step, lr7, eps_noise)
    dev = flat.device
    if out is None:
        out = dict(n_dead=torch.zeros(1, dtype=torch.int32, device=dev),
                   targets=torch.empty(G, dtype=torch.int32, device=dev))
    nbytes = lib().tts_relocate_workspace_bytes(G)
    ws = ws or Workspace(dev)
    buf = ws.get(nbytes)
    call("tts_sgld_relocate", ptr(flat), ptr(m), ptr(v), G, ptr(lr7), float(noise_lr), ptr(eps_noise),
         float(dead_thr), float(dead_frac), float(offset), ptr(targets_in), ptr(noise_in), ptr(step),
         int(seed) & (2 ** 64 - 1), ptr(out["n_dead"]), ptr(out["targets"]), ptr(buf), nbytes, stream())
    return out


def pack_operands(theta_u, color_o, o_col):
    _dev(theta_u, color_o, o_col)
    VT, K = theta_u.shape[0], theta_u.shape[2]
    slots = torch.empty(VT, K, SLOT_FLOATS, device=theta_u.device)
    call("tts_pack_operands", ptr(theta_u), ptr(color_o), ptr(o_col), VT, K, ptr(slots), stream())
    return slots


def unpack_slot_grads(slot_grads):
    _dev(slot_grads)
    VT, K = slot_grads.shape[0], slot_grads.shape[1]
    dev = slot_grads.device
    gth = torch.empty(VT, 6, K, device=dev)
    gcol = torch.empty(VT, K, 3, device=dev)
    goc = torch.empty(VT, K, 1, device=dev)
    call("tts_unpack_slot_grads", ptr(slot_grads), VT, K, ptr(gth), ptr(gcol), ptr(goc), stream())
    return gth, gcol, goc


def wsr_dense_fwd(theta_u, o, color, w_b, Phi, c_b, keep=None):
    _dev(theta_u, o, color, w_b, Phi, c_b, keep)
    P, G = Phi.shape[0], theta_u.shape[0]
    C = torch.empty(P, 3, device=Phi.device)
    den = torch.empty(P, device=Phi.device)
    call("tts_wsr_dense_fwd", ptr(theta_u), ptr(o), ptr(color), ptr(w_b), ptr(Phi), ptr(c_b), ptr(keep), P, G, ptr(C),
         ptr(den), stream())
    return C, den


def wsr_dense_bwd(theta_u, o, color, w_b, Phi, c_b, keep, C, den, gC):
    _dev(theta_u, o, color, w_b, Phi, c_b, keep, C, den, gC)
    P, G = Phi.shape[0], theta_u.shape[0]
    dev = Phi.device
    gth = torch.empty(G, 6, device=dev)
    go = torch.empty(G, device=dev)
    gcol = torch.empty(G, 3, device=dev)
    gwb = torch.empty(1, device=dev)
    call("tts_wsr_dense_bwd", ptr(theta_u), ptr(o), ptr(color), ptr(w_b), ptr(Phi), ptr(c_b), ptr(keep), P, G, ptr(C),
         ptr(den), ptr(gC), ptr(gth), ptr(go), ptr(gcol), ptr(gwb), stream())
    return gth, go, gcol, gwb


def unit_from_u8(src, out=None):
    """uint8 images -> float32 x / 255 (correctly rounded), same shape, on the device."""
    _dev(src, out)
    if src.dtype != torch.uint8:
        raise TypeError("unit_from_u8 takes a uint8 tensor")
    if out is None:
        out = torch.empty(src.shape, dtype=torch.float32, device=src.device)
    call("tts_unit_from_u8", ptr(src), src.numel(), ptr(out), stream())
    return out


def read_status():
    """Read and clear the device status word (bounded waits that gave up); synchronous."""
    import ctypes
    s = np.zeros(1, np.int32)
    call("tts_read_status", ctypes.c_void_p(s.ctypes.data))
    return int(s[0])


def peer_barrier(regions, phase, epoch):
    """tts_peer_barrier over the ranks of a PeerRegions (phase 0 or 1; epoch = device step)."""
    _dev(epoch)
    call("tts_peer_barrier", regions.t_flags, regions.rank, regions.world, int(phase), ptr(epoch), stream())


def peer_signal(regions, phase, epoch):
    _dev(epoch)
    call("tts_peer_signal", regions.t_flags, regions.rank, regions.world, int(phase), ptr(epoch), stream())


def peer_wait(regions, phase, epoch):
    _dev(epoch)
    call("tts_peer_wait", regions.t_flags, regions.rank, regions.world, int(phase), ptr(epoch), stream())


def adam_peer(regions, m, v, G, sh_degree, step, lr7, loss_total, betas=(0.9, 0.999), eps=1e-8):
    """tts_adam_peer: waits for every rank's gradient (phase 0), runs this rank's shard of the
    summed gradient through Adam, broadcasts it and signals phase 1."""
    _dev(m, v, step, lr7, loss_total)
    call("tts_adam_peer", regions.t_params, regions.t_grads, ptr(m), ptr(v), G, sh_degree, regions.rank,
         regions.world, ptr(step), ptr(lr7), float(betas[0]), float(betas[1]), float(eps), regions.t_loss,
         ptr(loss_total), regions.t_flags, stream())


def peer_sgld_relocate(regions, flat, m, v, G, step, lr7, noise_lr, eps_noise=None, dead_thr=0.005, dead_frac=0.0,
                       offset=0.0, seed=0, ws=None, out=None):
    """peer_sgld(...) then relocate(...) in one launch (waits for phase 1 like peer_sgld)."""
    _dev(flat, m, v, step, lr7, eps_noise)
    dev = flat.device
    if out is None:
        out = dict(n_dead=torch.zeros(1, dtype=torch.int32, device=dev),
                   targets=torch.empty(G, dtype=torch.int32, device=dev))
    nbytes = lib().tts_relocate_workspace_bytes(G)
    ws = ws or Workspace(dev)
    buf = ws.get(nbytes)
    call("tts_peer_sgld_relocate", ptr(flat), ptr(m), ptr(v), G, ptr(lr7), float(noise_lr), ptr(eps_noise),
         float(dead_thr), float(dead_frac), float(offset), ptr(step), int(seed) & (2 ** 64 - 1), ptr(out["n_dead"]),
         ptr(out["targets"]), regions.t_flags, regions.rank, regions.world, ptr(buf), nbytes, stream())
    return out


def peer_sgld(regions, flat, G, step, lr_means, noise_lr, eps_noise=None, seed=0):
    """SGLD once every rank's update has arrived (phase 1)."""
    _dev(flat, step, eps_noise)
    call("tts_peer_sgld", ptr(flat), G, float(lr_means), float(noise_lr), ptr(eps_noise), ptr(step),
         int(seed) & (2 ** 64 - 1), regions.t_flags, regions.rank, regions.world, stream())



# ---- the composable spike API (spike/geometry.py, spike/sh.py, spike/forward.py) --------------
# fp32 or fp64 tensors on the current CUDA device; outputs allocated here with the inputs' dtype.
_SPIKE_DTYPES = {torch.float32: 0, torch.float64: 1}


def spike_dtype(*ts):
    """dtype code (0 float32, 1 float64) shared by the given tensors; raises for CPU tensors,
    other dtypes or mixed dtypes (the reference's functions compute in their inputs' dtype)."""
    ts = [t for t in ts if t is not None]
    _dev(*ts)
    dt = ts[0].dtype
    if dt not in _SPIKE_DTYPES or any(t.dtype != dt for t in ts):
        raise TypeError(f"spike ops take float32 or float64 tensors of one dtype, got {[t.dtype for t in ts]}")
    return _SPIKE_DTYPES[dt]


def _cam16(R_v, t_v, fx, fy, cx, cy):
    """Host double[16] camera record: R_v (row-major), t_v, fx, fy, cx, cy (constants)."""
    import ctypes
    vals = [float(x) for x in torch.as_tensor(R_v).detach().reshape(-1).cpu().tolist()]
    vals += [float(x) for x in torch.as_tensor(t_v).detach().reshape(-1).cpu().tolist()]
    vals += [float(torch.as_tensor(x).item()) if torch.is_tensor(x) else float(x) for x in (fx, fy, cx, cy)]
    if len(vals) != 16:
        raise ValueError("R_v must be 3x3 and t_v of length 3")
    return (ctypes.c_double * 16)(*vals)


def quat_to_rotmat(q):
    dt = spike_dtype(q)
    n = q.numel() // 4
    R = torch.empty(q.shape[:-1] + (3, 3), dtype=q.dtype, device=q.device)
    call("tts_quat_to_rotmat", ptr(q), n, ptr(R), dt, stream())
    return R


def quat_to_rotmat_bwd(q, gR):
    dt = spike_dtype(q, gR)
    gq = torch.empty_like(q)
    call("tts_quat_to_rotmat_bwd", ptr(q), ptr(gR), q.numel() // 4, ptr(gq), dt, stream())
    return gq


def cov3d(s, R):
    dt = spike_dtype(s, R)
    cov = torch.empty_like(R)
    call("tts_cov3d", ptr(s), ptr(R), s.numel() // 3, ptr(cov), dt, stream())
    return cov


def cov3d_bwd(s, R, gcov):
    dt = spike_dtype(s, R, gcov)
    gs, gR = torch.empty_like(s), torch.empty_like(R)
    call("tts_cov3d_bwd", ptr(s), ptr(R), ptr(gcov), s.numel() // 3, ptr(gs), ptr(gR), dt, stream())
    return gs, gR


def project_ewa(means, cov, cam16, blur, near):
    dt = spike_dtype(means, cov)
    G = means.shape[0]
    o = lambda *shape: torch.empty(shape, dtype=means.dtype, device=means.device)  # noqa: E731
    mu2d, conic, depth = o(G, 2), o(G, 3), o(G)
    keep = torch.empty(G, dtype=torch.uint8, device=means.device)
    call("tts_project_ewa", ptr(means), ptr(cov), G, cam16, float(blur), float(near), ptr(mu2d), ptr(conic),
         ptr(depth), ptr(keep), dt, stream())
    return mu2d, conic, depth, keep.view(torch.bool)


def project_ewa_bwd(means, cov, cam16, blur, near, gmu2d, gconic, gdepth):
    dt = spike_dtype(means, cov, gmu2d, gconic, gdepth)
    gm, gc = torch.empty_like(means), torch.empty_like(cov)
    call("tts_project_ewa_bwd", ptr(means), ptr(cov), means.shape[0], cam16, float(blur), float(near), ptr(gmu2d),
         ptr(gconic), ptr(gdepth), ptr(gm), ptr(gc), dt, stream())
    return gm, gc


def eval_sh(deg, coeffs, dirs, raw=False):
    dt = spike_dtype(coeffs, dirs)
    G = dirs.numel() // 3
    nc, nch = coeffs.shape[-2], coeffs.shape[-1]
    out = torch.empty(dirs.shape[:-1] + (nch,), dtype=dirs.dtype, device=dirs.device)
    call("tts_eval_sh", int(deg), ptr(coeffs), nc, nch, ptr(dirs), G, int(bool(raw)), ptr(out), dt, stream())
    return out


def eval_sh_bwd(deg, coeffs, dirs, gout, raw=False):
    dt = spike_dtype(coeffs, dirs, gout)
    gco, gd = torch.empty_like(coeffs), torch.empty_like(dirs)
    call("tts_eval_sh_bwd", int(deg), ptr(coeffs), coeffs.shape[-2], coeffs.shape[-1], ptr(dirs), dirs.numel() // 3,
         int(bool(raw)), ptr(gout), ptr(gco), ptr(gd), dt, stream())
    return gco, gd


def color_from_dc(dc, gout=None):
    dt = spike_dtype(dc, gout)
    out = torch.empty_like(dc)
    call("tts_color_from_dc", ptr(dc), dc.numel(), ptr(gout), ptr(out), dt, stream())
    return out


def phi(px, py):
    dt = spike_dtype(px, py)
    out = torch.empty(px.numel(), 6, dtype=px.dtype, device=px.device)
    call("tts_phi", ptr(px), ptr(py), px.numel(), ptr(out), dt, stream())
    return out


def phi_bwd(px, py, gPhi):
    dt = spike_dtype(px, py, gPhi)
    gx, gy = torch.empty_like(px), torch.empty_like(py)
    call("tts_phi_bwd", ptr(px), ptr(py), ptr(gPhi), px.numel(), ptr(gx), ptr(gy), dt, stream())
    return gx, gy


def theta_from_conic(conic, mu, k, origins=None, per=1, gathered=False, want_Q=True, want_u=True):
    """theta_Q / theta_u [n,6] (layout of spike/forward.py:23-39), or with ``gathered`` theta_u
    as [n/per, 6, per] in the op order of theta_u_gathered (tools/m4_train_binned.py:130-143);
    the means are taken relative to ``origins[i // per]`` when given."""
    dt = spike_dtype(conic, mu, origins)
    n = conic.numel() // 3
    o = lambda *shape: torch.empty(shape, dtype=conic.dtype, device=conic.device)  # noqa: E731
    if gathered:
        thQ, thU = None, o(n // per, 6, per)
    else:
        thQ, thU = (o(n, 6) if want_Q else None), (o(n, 6) if want_u else None)
    call("tts_theta_from_conic", ptr(conic), ptr(mu), ptr(origins), int(per), n, float(k), 1 if gathered else 0,
         ptr(thQ), ptr(thU), dt, stream())
    return thQ, thU


def theta_from_conic_bwd(conic, mu, k, gQ, gU, origins=None, per=1):
    dt = spike_dtype(conic, mu, origins, gQ, gU)
    gc, gm = torch.empty_like(conic), torch.empty_like(mu)
    call("tts_theta_from_conic_bwd", ptr(conic), ptr(mu), ptr(origins), int(per), conic.numel() // 3, float(k),
         ptr(gQ), ptr(gU), ptr(gc), ptr(gm), dt, stream())
    return gc, gm


def _spike_ws(P, G, dt, device):
    nbytes = lib().tts_spike_workspace_bytes(int(P), int(G), int(dt))
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device), nbytes


def quad_form(px, py, mu2d, conic):
    dt = spike_dtype(px, py, mu2d, conic)
    P, G = px.numel(), mu2d.shape[0]
    Q = torch.empty(P, G, dtype=px.dtype, device=px.device)
    call("tts_quad_form", ptr(px), ptr(py), ptr(mu2d), ptr(conic), P, G, ptr(Q), dt, stream())
    return Q


def quad_form_bwd(px, py, mu2d, conic, gQ):
    dt = spike_dtype(px, py, mu2d, conic, gQ)
    P, G = px.numel(), mu2d.shape[0]
    gm, gc = torch.empty_like(mu2d), torch.empty_like(conic)
    ws, nbytes = _spike_ws(P, G, dt, px.device)
    call("tts_quad_form_bwd", ptr(px), ptr(py), ptr(mu2d), ptr(conic), ptr(gQ), P, G, ptr(gm), ptr(gc), ptr(ws), nbytes,
         dt, stream())
    return gm, gc


def phi_theta(Phi, theta):
    dt = spike_dtype(Phi, theta)
    P, G = Phi.shape[0], theta.shape[0]
    Q = torch.empty(P, G, dtype=Phi.dtype, device=Phi.device)
    call("tts_phi_theta", ptr(Phi), ptr(theta), P, G, ptr(Q), dt, stream())
    return Q


def phi_theta_bwd(Phi, theta, gQ, want_phi=True, want_theta=True):
    dt = spike_dtype(Phi, theta, gQ)
    P, G = Phi.shape[0], theta.shape[0]
    gP = torch.empty_like(Phi) if want_phi else None
    gT = torch.empty_like(theta) if want_theta else None
    ws, nbytes = _spike_ws(P, G, dt, Phi.device)
    call("tts_phi_theta_bwd", ptr(Phi), ptr(theta), ptr(gQ), P, G, ptr(gP), ptr(gT), ptr(ws), nbytes, dt, stream())
    return gP, gT


def poly_splat_wgeo(Q, k, keep=None, gout=None):
    dt = spike_dtype(Q, gout)
    _dev(keep)
    P, G = Q.shape[0], Q.shape[1]
    out = torch.empty_like(Q)
    call("tts_poly_splat_wgeo", ptr(Q), P, G, float(k), ptr(keep), ptr(gout), ptr(out), dt, stream())
    return out


def fp32_peak_tflops(reps=5, iters=4096):
    """Measured FP32 FMA-pipe peak (TFLOP/s) of the current device: the best of ``reps`` timed
    launches of the packed-FMA probe kernel (CUDA events on the current stream)."""
    dev = torch.cuda.current_device()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks = sms * 8
    out = torch.empty(blocks * 256, device="cuda")
    flops = lib().tts_fma_probe_flops(blocks, iters)
    call("tts_fma_probe", blocks, iters, ptr(out), stream())        # warm-up
    best = 0.0
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        call("tts_fma_probe", blocks, iters, ptr(out), stream())
        e1.record()
        e1.synchronize()
        best = max(best, flops / (e0.elapsed_time(e1) * 1e-3) / 1e12)
    return best
