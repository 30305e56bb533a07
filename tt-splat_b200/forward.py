"""The per-pixel forward primitives of the matrix-native splat (spike/forward.py:13-71) on the device.

Each function keeps the reference's signature and is a torch autograd Function over a forward
and a backward kernel of ``libttsplat_b200.so`` (float32 or float64; CPU tensors raise):

* ``quad_form(px, py, mu2d, conic_abc)`` -> Q [P,G], the raw Mahalanobis form
  a dx^2 + 2 b dx dy + c dy^2 of every pixel centre against every gaussian (no /k);
* ``theta_from_conic(conic_abc, mu2d, k)`` -> (theta_Q [G,6], theta_u [G,6]): the coefficients of
  Q and of u = 1 - Q/k over the monomials Phi = [px^2, py^2, px py, px, py, 1];
* ``phi(px, py)`` -> Phi [P,6];
* ``quad_form_tilelocal(lx, ly, conic_abc, mu2d, tile_origin)`` -> Q [P,G] as the GEMM
  Phi(lx, ly) theta_Q^T with the tile origin folded into the means (tile-local pixel
  coordinates keep the monomials small, which is what makes the low-precision form usable);
* ``poly_splat_wgeo(Q, k, keep)`` -> max(0, 1 - Q/k)^2, zero for culled gaussians;
* ``color_from_dc(color_dc)`` -> clamp(0.5 + C0 dc, min 0).

Pixel grids and tile origins are constants (no gradient), as in the reference's renders.  The
fused tile kernels evaluate the same algebra per tile and never materialise Q; these are the
building blocks for callers that compose the dense form by hand.
"""
import torch

from . import ops
from ._lib import on_device


def _c(t):
    return t.detach().contiguous()


class _QuadForm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, px, py, mu2d, conic):
        a = [_c(px).reshape(-1), _c(py).reshape(-1), _c(mu2d), _c(conic)]
        ctx.save_for_backward(*a)
        return ops.quad_form(*a)

    @staticmethod
    def backward(ctx, gQ):
        px, py, mu2d, conic = ctx.saved_tensors
        gm, gc = ops.quad_form_bwd(px, py, mu2d, conic, gQ.contiguous())
        return None, None, gm, gc


class _Theta(torch.autograd.Function):
    """theta_Q and theta_u of conic/means (the means relative to one origin when given)."""

    @staticmethod
    def forward(ctx, conic, mu2d, k, origin):
        c, m = _c(conic), _c(mu2d)
        o = None if origin is None else _c(origin).reshape(-1).to(c.dtype)
        thQ, thU = ops.theta_from_conic(c, m, k, origins=o, per=max(c.shape[0], 1))
        ctx.save_for_backward(c, m)
        ctx.k, ctx.origin = k, o
        return thQ, thU

    @staticmethod
    def backward(ctx, gQ, gU):
        c, m = ctx.saved_tensors
        f = lambda g: None if g is None else g.contiguous()  # noqa: E731
        gc, gm = ops.theta_from_conic_bwd(c, m, ctx.k, f(gQ), f(gU), origins=ctx.origin, per=max(c.shape[0], 1))
        return gc, gm, None, None


class _Phi(torch.autograd.Function):
    @staticmethod
    def forward(ctx, px, py):
        x, y = _c(px).reshape(-1), _c(py).reshape(-1)
        ctx.save_for_backward(x, y)
        ctx.shapes = (px.shape, py.shape)
        return ops.phi(x, y)

    @staticmethod
    def backward(ctx, gPhi):
        x, y = ctx.saved_tensors
        gx, gy = ops.phi_bwd(x, y, gPhi.contiguous())
        return gx.reshape(ctx.shapes[0]), gy.reshape(ctx.shapes[1])


class _PhiTheta(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Phi, theta):
        p, t = _c(Phi), _c(theta)
        ctx.save_for_backward(p, t)
        return ops.phi_theta(p, t)

    @staticmethod
    def backward(ctx, gQ):
        p, t = ctx.saved_tensors
        gP, gT = ops.phi_theta_bwd(p, t, gQ.contiguous(), want_phi=ctx.needs_input_grad[0],
                                   want_theta=ctx.needs_input_grad[1])
        return gP, gT


class _PolySplat(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, k, keep):
        q = _c(Q)
        kp = None if keep is None else keep.detach().to(torch.uint8).contiguous()
        ctx.save_for_backward(q)
        ctx.k, ctx.keep = k, kp
        return ops.poly_splat_wgeo(q, k, kp)

    @staticmethod
    def backward(ctx, g):
        (q,) = ctx.saved_tensors
        return ops.poly_splat_wgeo(q, ctx.k, ctx.keep, gout=g.contiguous()), None, None


class _ColorDC(torch.autograd.Function):
    @staticmethod
    def forward(ctx, dc):
        d = _c(dc)
        ctx.save_for_backward(d)
        return ops.color_from_dc(d)

    @staticmethod
    def backward(ctx, g):
        (d,) = ctx.saved_tensors
        return ops.color_from_dc(d, gout=g.contiguous())


def quad_form(px, py, mu2d, conic_abc):
    """px, py [P]; mu2d [G,2]; conic_abc [G,3] -> Q [P,G] (spike/forward.py:13-20)."""
    with on_device(mu2d):
        return _QuadForm.apply(px, py, mu2d, conic_abc)


def theta_from_conic(conic_abc, mu2d, k):
    """-> (theta_Q [G,6], theta_u [G,6]) over Phi (spike/forward.py:23-39)."""
    with on_device(conic_abc):
        return _Theta.apply(conic_abc, mu2d, float(k), None)


def phi(px, py):
    """Monomial basis [P,6] of the pixel coordinates (spike/forward.py:42-44)."""
    with on_device(px):
        return _Phi.apply(px, py)


def quad_form_tilelocal(lx, ly, conic_abc, mu2d, tile_origin):
    """Q [P,G] over one tile as Phi(lx, ly) theta_Q^T with mu_local = mu2d - tile_origin
    (spike/forward.py:47-58); lx, ly are tile-local pixel coordinates."""
    with on_device(mu2d):
        Phi = _Phi.apply(lx, ly)
        theta_Q, _ = _Theta.apply(conic_abc, mu2d, 1.0, torch.as_tensor(tile_origin, device=mu2d.device))
        return _PhiTheta.apply(Phi, theta_Q)


def poly_splat_wgeo(Q, k, keep=None):
    """max(0, 1 - Q/k)^2 [P,G], times keep [G] when given (spike/forward.py:61-66)."""
    with on_device(Q):
        return _PolySplat.apply(Q, float(k), keep)


def color_from_dc(color_dc):
    """clamp(0.5 + C0 dc, min 0) (spike/forward.py:69-71)."""
    with on_device(color_dc):
        return _ColorDC.apply(color_dc)
