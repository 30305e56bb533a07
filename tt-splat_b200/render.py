"""End-to-end binned render: gaussian model + camera(s) -> image(s) (mirrors spike/render.py:14-49).

``render(model, cam, arm="A", k, blur_eps, near, sh_degree)`` keeps the reference signature and
runs the B200 path: the fused projection kernel (geometry + SH colour + activations), the
bit-exact binning with its slot-row pack, and the fused per-tile forward.  It is differentiable:
the backward runs the fused per-tile backward and the parameter backward kernel, returning the
gradient of every model parameter.  Rendering is binned (16x16 tiles, radius-R neighbour cells,
K gaussians per tile, the reference's ``tools/m4_train_binned.py`` operator), which equals the
dense ``spike.render`` whenever no tile overflows K and no gaussian reaches past its stencil.
Arms A (plain weighted-sum rendering), B (opacity scaled by the depth weight
sigmoid(depth_beta (depth_tau - z)), spike/arms.py:34-37) and RV (revealage compositing
C = Cavg (1 - R) + c_b R, spike/arms.py:70-83) are on this path.
"""
import torch

from . import ops
from ._lib import on_device, require_cuda
from .camera import as_camera, pack_cameras
from .model import flat_of

ARMS = ("A", "B", "C0", "C", "SZ", "RV", "D")


class _BinnedRender(torch.autograd.Function):
    @staticmethod
    def forward(ctx, flat, depth_bt, cams_t, c_b, cfg):
        G, sh_degree, H, W, R, K, k, blur, near, bf16, rv = cfg
        flat_d = flat.detach().contiguous()
        bt = depth_bt.detach().float().contiguous() if depth_bt is not None else None
        need_grad = ctx.needs_input_grad[0] or (depth_bt is not None and ctx.needs_input_grad[1])
        pj = ops.project(flat_d, G, sh_degree, cams_t, H, W, blur, near, depth_bt=bt)
        if bf16 and not need_grad:
            bp = ops.bin_pack(pj, G, H, W, R, K, k, with_inv=False, bf16=True)
            slots = bp["slots"]
        else:
            # the backward always works on fp32 slot rows; the bf16 forward gets its own compact rows
            bp = ops.bin_pack(pj, G, H, W, R, K, k, with_inv=need_grad)
            slots = ops.bin_pack(pj, G, H, W, R, K, k, with_inv=False, bf16=True)["slots"] if bf16 else bp["slots"]
        if rv:
            rf = ops.render_fwd_rv(slots, bp["count"], H, W, c_b)
            keep = rf["aux"]                       # (Cavg, R) per pixel in place of the image
        else:
            rf = ops.render_fwd(slots, bp["count"], H, W, flat_d[59 * G:], c_b, bf16=bf16)
            keep = rf["img"]
        ctx.save_for_backward(flat_d, cams_t, c_b, bp["slots"], bp["count"], bp["inv"], keep, rf["den"],
                              pj["proj"])
        ctx.cfg = cfg
        ctx.bt = bt
        ctx.bins = bp
        return rf["img"]

    @staticmethod
    def backward(ctx, gimg):
        flat, cams_t, c_b, slots, count, inv, img_or_aux, den, proj = ctx.saved_tensors
        G, sh_degree, H, W, R, K, k, blur, near, _, rv = ctx.cfg
        if rv:
            rb = ops.render_bwd_rv(slots, count, H, W, c_b, den, img_or_aux, gimg.contiguous())
        else:
            rb = ops.render_bwd(slots, count, H, W, c_b, img_or_aux, den, gimg.contiguous())
        out = ops.backward_params(flat, G, sh_degree, cams_t, H, W, R, K, inv, rb["slot_grads"], rb["gwb"], k, blur, near,
                                  proj=proj, depth_bt=ctx.bt)
        if ctx.bt is None:
            return out, None, None, None, None
        grads, gbt = out
        return grads, gbt, None, None, None


def render_views(model, cams, k=4.0, blur_eps=0.3, near=0.2, sh_degree=0, R=1, K=128, bf16=False, arm="A"):
    """Render V views in one batched launch per stage -> [V, H, W, 3] (arm A; arm B with the
    model's depth_beta / depth_tau; arm RV, revealage compositing, fp32 rows)."""
    if arm == "RV" and bf16:
        raise NotImplementedError("bf16 slot rows are implemented for arms A and B")
    require_cuda()
    cams = [as_camera(c) for c in cams]
    flat = flat_of(model)
    if not flat.is_cuda:
        raise RuntimeError("the model must live on a CUDA device (no CPU fallback)")
    G = model.means3d.shape[0]
    H, W = cams[0].H, cams[0].W
    ops.tiles(H, W)
    cams_t = pack_cameras(cams, flat.device)
    c_b = getattr(model, "c_b", None)
    c_b = torch.ones(3, device=flat.device) if c_b is None else c_b.to(flat.device).float().contiguous()
    cfg = (G, int(sh_degree), H, W, int(R), int(K), float(k), float(blur_eps), float(near), bool(bf16), arm == "RV")
    depth_bt = None
    if arm == "B":
        depth_bt = torch.stack([torch.as_tensor(model.depth_beta), torch.as_tensor(model.depth_tau)]).float()
        depth_bt = depth_bt.to(flat.device)
    with on_device(flat):
        return _BinnedRender.apply(flat, depth_bt, cams_t, c_b, cfg)


def render(model, cam, arm="A", k=4.0, blur_eps=0.3, near=0.2, sh_degree=0, R=1, K=128, bf16=False):
    """spike/render.py:14-49 on the B200 path -> [H, W, 3]."""
    if arm not in ARMS:
        raise ValueError(f"unknown arm {arm!r}")
    if arm not in ("A", "B", "RV"):
        raise NotImplementedError(f"arm {arm!r} is not on the B200 hot path (arms A, B and RV)")
    return render_views(model, [cam], k, blur_eps, near, sh_degree, R, K, bf16, arm=arm)[0]
