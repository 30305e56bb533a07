"""The binned render operator pair of tools/m4_train_binned.py on the B200 kernels.

- ``TileMap`` (:60-72), ``assign_bins`` (:75-127, canonical stable order, bit-exact),
  ``theta_u_gathered`` (:130-143, the theta kernel in that function's op order, differentiable);
- ``_operands(model, cam, tmap, R, K)`` (:189-212): geometry, activations, binning and the
  per-tile operand gather, differentiable in the model parameters;
- ``_DevRenderBinned.apply(theta_u, color_o, o_col, w_b, Phi, gidx, c_b, H, W)`` (:154-186):
  the per-tile WSR forward and backward on operands in the reference's layout.
"""
import torch

from ._lib import on_device
from . import ops
from .camera import as_camera, pack_cameras
from .model import flat_of

K_POLY = 4.0


class TileMap:
    """tools/m4_train_binned.py:60-72."""

    def __init__(self, H, W, device="cuda"):
        assert H % 16 == 0 and W % 16 == 0
        self.H, self.W, self.nty, self.ntx = H, W, H // 16, W // 16
        self.T = self.nty * self.ntx
        p = torch.arange(256)
        # the monomials [x^2, y^2, x y, x, y, 1] of the 256 tile-local pixel centres (a constant
        # table of the tile map; the tile kernels generate the same values in registers)
        lx, ly = (p % 16).float() + 0.5, (p // 16).float() + 0.5
        self.Phi = torch.stack([lx * lx, ly * ly, lx * ly, lx, ly, torch.ones(256)], dim=1).to(device)
        t = torch.arange(self.T)
        ty, tx = t // self.ntx, t % self.ntx
        self.origins = torch.stack([(tx * 16).float(), (ty * 16).float()], dim=1).to(device)
        gr = ty[:, None] * 16 + (p // 16)[None, :]
        gc = tx[:, None] * 16 + (p % 16)[None, :]
        self.gidx = (gr * W + gc).reshape(-1).long().to(device)


def bin_tables(mu2d, keep, tmap, R=1, K=128):
    """Device binning tables for mu2d[G,2] (or [V,G,2]): idx (int32, -1 unused), count, cand,
    and the stencil-indexed inverse table."""
    idx, count, cand, inv = ops.bin_from_mu2d(mu2d, keep, tmap.H, tmap.W, R, K)
    return dict(idx=idx, count=count, cand=cand, inv=inv)


@torch.no_grad()
def assign_bins(mu2d, keep, tmap, R, K):
    """tools/m4_train_binned.py:75-127 -> idx[T,K] long (0 in invalid slots), valid[T,K] bool."""
    idx, _, _, _ = ops.bin_from_mu2d(mu2d.detach(), keep.detach(), tmap.H, tmap.W, R, K, with_inv=False)
    idx = idx[0]
    valid = idx >= 0
    return torch.where(valid, idx, torch.zeros_like(idx)).long(), valid


class _ThetaGathered(torch.autograd.Function):
    @staticmethod
    def forward(ctx, conic_t, mu_t, origins, k):
        T, K = conic_t.shape[0], conic_t.shape[1]
        c = conic_t.detach().contiguous().reshape(T * K, 3)
        m = mu_t.detach().contiguous().reshape(T * K, 2)
        o = origins.detach().to(c.dtype).contiguous()
        _, th = ops.theta_from_conic(c, m, k, origins=o, per=K, gathered=True)
        ctx.save_for_backward(c, m, o)
        ctx.k, ctx.TK = k, (T, K)
        return th

    @staticmethod
    def backward(ctx, g):
        c, m, o = ctx.saved_tensors
        T, K = ctx.TK
        gU = g.transpose(1, 2).contiguous().reshape(T * K, 6)
        gc, gm = ops.theta_from_conic_bwd(c, m, ctx.k, None, gU, origins=o, per=K)
        return gc.reshape(T, K, 3), gm.reshape(T, K, 2), None, None


def theta_u_gathered(conic_t, mu_t, origins, k):
    """tools/m4_train_binned.py:130-143: conic_t [T,K,3], mu_t [T,K,2] (global), origins [T,2]
    -> theta_u [T,6,K] with each tile's origin folded into the means, on the device in the
    reference function's op order; differentiable in conic_t and mu_t."""
    with on_device(conic_t):
        return _ThetaGathered.apply(conic_t, mu_t, origins, float(k))


class _Operands(torch.autograd.Function):
    @staticmethod
    def forward(ctx, flat, cams_t, cached_idx, cfg):
        G, sh_degree, H, W, R, K, k, blur, near = cfg
        flat_d = flat.detach().contiguous()
        pj = ops.project(flat_d, G, sh_degree, cams_t, H, W, blur, near)
        if cached_idx is None:
            bp = ops.bin_pack(pj, G, H, W, R, K, k)
        else:
            bp = ops.pack_cached(pj, G, H, W, R, K, cached_idx, k)
        idx = bp["idx"][0]
        valid = idx >= 0
        # the kernels write only the valid slots' rows; the operands are zero elsewhere, like the
        # reference's products with valid (tools/m4_train_binned.py:209-211)
        s = torch.where(valid[..., None], bp["slots"][0], torch.zeros((), device=flat_d.device))   # [T,K,12]
        theta_u = s[..., 0:6].transpose(1, 2).contiguous()
        color_o = s[..., 6:9].contiguous()
        o_col = s[..., 9:10].contiguous()
        w_b = torch.nn.functional.softplus(flat_d[59 * G])
        ctx.save_for_backward(flat_d, cams_t, bp["inv"])
        ctx.cfg = cfg
        ctx.mark_non_differentiable(idx, valid)
        return theta_u, color_o, o_col, w_b, torch.where(valid, idx, torch.zeros_like(idx)).long(), valid

    @staticmethod
    def backward(ctx, gth, gcol, goc, gwb, _gi, _gv):
        flat, cams_t, inv = ctx.saved_tensors
        G, sh_degree, H, W, R, K, k, blur, near = ctx.cfg
        T = (H // 16) * (W // 16)
        dev = flat.device
        z = lambda t, shp: torch.zeros(shp, device=dev) if t is None else t.float()  # noqa: E731
        gth, gcol, goc = z(gth, (T, 6, K)), z(gcol, (T, K, 3)), z(goc, (T, K, 1))
        sg = torch.cat([gth.transpose(1, 2), gcol, goc], -1).contiguous()[None]     # [1,T,K,10]
        part = torch.zeros(1, T, device=dev)
        if gwb is not None:
            part[0, 0] = gwb
        grads = ops.backward_params(flat, G, sh_degree, cams_t, H, W, R, K, inv, sg, part, k, blur, near)
        return grads, None, None, None


def _cached_table(cached_bins, G, T, K, device):
    """The reference's (idx, valid) pair -> int32 [1,T,K] ids with -1 where invalid; the valid
    slots of a tile must come first (as assign_bins writes them)."""
    idx, valid = cached_bins
    idx = torch.as_tensor(idx, device=device)
    valid = torch.as_tensor(valid, device=device).bool()
    if tuple(idx.shape) != (T, K) or tuple(valid.shape) != (T, K):
        raise ValueError(f"cached_bins must be ([{T}, {K}], [{T}, {K}]) tables")
    if bool((valid[:, 1:] & ~valid[:, :-1]).any()):
        raise ValueError("cached_bins: the valid slots of a tile must come first")
    if bool(((idx < 0) | (idx >= G))[valid].any()):
        raise ValueError("cached_bins: gaussian ids out of range")
    return torch.where(valid, idx, torch.full_like(idx, -1)).to(torch.int32).contiguous()[None]


def _operands(model, cam, tmap, R, K, cached_bins=None, sh_degree=0, blur=0.3, near=0.2):
    """tools/m4_train_binned.py:189-212 -> (theta_u[T,6,K], color_o_t[T,K,3], o_col_t[T,K,1], w_b,
    (idx, valid)).  The colour is the SH colour of degree ``sh_degree`` (0 = the reference's DC).
    With ``cached_bins`` (an (idx, valid) pair from an earlier call) the binning is skipped: the
    operands of the current parameters are gathered through those tables, and the pair is
    returned as given."""
    cam = as_camera(cam)
    flat = flat_of(model)
    G = model.means3d.shape[0]
    cfg = (G, int(sh_degree), cam.H, cam.W, int(R), int(K), K_POLY, float(blur), float(near))
    with on_device(flat):
        cached = None if cached_bins is None else _cached_table(cached_bins, G, tmap.T, int(K), flat.device)
        th, col, oc, w_b, idx, valid = _Operands.apply(flat, pack_cameras([cam], flat.device), cached, cfg)
    if cached_bins is not None:
        return th, col, oc, w_b, cached_bins
    return th, col, oc, w_b, (idx, valid)


class _DevRenderBinned(torch.autograd.Function):
    """tools/m4_train_binned.py:154-186: render from per-tile operands; grads for the first four."""

    @staticmethod
    def forward(ctx, theta_u, color_o, o_col, w_b, Phi, gidx, c_b, H, W):
        T, K = theta_u.shape[0], theta_u.shape[2]
        assert Phi.shape == (256, 6) and gidx.numel() == T * 256, "standard 16x16 TileMap operands expected"
        slots = ops.pack_operands(theta_u.detach().float().contiguous(), color_o.detach().float().contiguous(),
                                  o_col.detach().float().contiguous())[None]
        count = torch.full((1, T), K, dtype=torch.int32, device=theta_u.device)
        wb = torch.as_tensor(w_b, dtype=torch.float32, device=theta_u.device).detach().reshape(1).contiguous()
        cb = c_b.detach().float().contiguous().to(theta_u.device)
        rf = ops.render_fwd(slots, count, H, W, wb, cb, w_b_is_raw=False)
        ctx.save_for_backward(slots, count, cb, rf["img"], rf["den"])
        ctx.shape = (H, W, torch.as_tensor(w_b).shape)
        return rf["img"][0]

    @staticmethod
    def backward(ctx, gimg):
        slots, count, cb, img, den = ctx.saved_tensors
        H, W, wshape = ctx.shape
        rb = ops.render_bwd(slots, count, H, W, cb, img, den, gimg.float().contiguous()[None])
        gth, gcol, goc = ops.unpack_slot_grads(rb["slot_grads"][0])
        return gth, gcol, goc, rb["gwb"].sum().reshape(wshape), None, None, None, None, None


def render_binned_device(model, cam, tmap, R=1, K=128, cached_bins=None, return_bins=False, sh_degree=0):
    """tools/m4_train_binned.py:215-219: the image [H, W, 3], and with ``return_bins`` the (idx,
    valid) pair the binning produced (or ``cached_bins``, which skips the binning)."""
    thU, col, oc, w_b, bins = _operands(model, cam, tmap, R, K, cached_bins=cached_bins, sh_degree=sh_degree)
    c_b = getattr(model, "c_b", torch.ones(3, device=thU.device))
    with on_device(thU):
        img = _DevRenderBinned.apply(thU, col, oc, w_b, tmap.Phi, tmap.gidx, c_b, tmap.H, tmap.W)
    return (img, bins) if return_bins else img
