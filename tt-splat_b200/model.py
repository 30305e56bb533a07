"""The gaussian set as one flat device buffer (mirrors spike/model.py:16-95).

All per-gaussian parameters live in a single fp32 tensor ``flat[59*G + 1]`` in the layout the
kernels read (``include/ttsplat_b200.h``): means3d[G,3] | log_scales[G,3] | quats[G,4] |
opacity_raw[G] | color_dc[G,3] | color_rest[G,15,3] | w_b_raw.  The reference's attribute
names are views into it, so code written against ``spike.model.GaussianModel`` reads the same
fields.  The fused Adam keeps its moments in buffers of the same layout.
"""
import math

import numpy as np
import torch
import torch.nn as nn

C0 = 0.28209479177387814
NAMES = ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest")
WIDTHS = {"means3d": 3, "log_scales": 3, "quats": 4, "opacity_raw": 1, "color_dc": 3, "color_rest": 45}
SHAPES = {"means3d": (3,), "log_scales": (3,), "quats": (4,), "opacity_raw": (), "color_dc": (3,),
          "color_rest": (15, 3)}


def offsets(G):
    off, o = {}, 0
    for n in NAMES:
        off[n] = (o, o + WIDTHS[n] * G)
        o += WIDTHS[n] * G
    off["w_b_raw"] = (o, o + 1)
    return off


def flat_size(G):
    return 59 * G + 1


def view(flat, G, name):
    a, b = offsets(G)[name]
    if name == "w_b_raw":
        return flat[a:b].reshape(())
    return flat[a:b].view((G,) + SHAPES[name])


def pack_arrays(params, device=None):
    """dict of numpy/torch arrays (reference field names) -> flat fp32 tensor."""
    G = int(np.asarray(params["means3d"]).shape[0])
    parts = []
    for n in NAMES:
        x = params.get(n)
        if x is None:
            x = np.zeros((G,) + SHAPES[n], np.float32)
        parts.append(torch.as_tensor(np.asarray(x, np.float32) if not torch.is_tensor(x) else x.detach().cpu().float()).reshape(-1))
    parts.append(torch.as_tensor(np.float32(params["w_b_raw"])).reshape(1))
    return torch.cat(parts).to(device)


class GaussianModel(nn.Module):
    """spike/model.py:16-95 with a flat parameter buffer.  The initial values are drawn with the
    same generator calls in the same order as the reference, so a seed gives the same model."""

    def __init__(self, G, extent=1.3, dtype=torch.float32, device="cuda", seed=0, gt=False, init_scale=0.05,
                 depth_tau=3.0, _flat=None):
        super().__init__()
        self.G_ = int(G)
        if _flat is None:
            g = torch.Generator(device="cpu").manual_seed(seed)

            def rand(*s):
                return torch.rand(*s, generator=g, dtype=torch.float32)

            def randn(*s):
                return torch.randn(*s, generator=g, dtype=torch.float32)
            means = (rand(G, 3) * 2 - 1) * extent
            ls = torch.full((G, 3), math.log(init_scale)) + 0.1 * randn(G, 3)
            q = torch.zeros(G, 4)
            q[:, 0] = 1.0
            q = q + 0.1 * randn(G, 4)
            o0 = 0.7 if gt else 0.1
            op = torch.full((G,), math.log(o0 / (1 - o0)))
            dc = (randn(G, 3) * 1.5) if gt else (0.01 * randn(G, 3))
            _flat = pack_arrays(dict(means3d=means, log_scales=ls, quats=q, opacity_raw=op, color_dc=dc,
                                     color_rest=torch.zeros(G, 15, 3), w_b_raw=-3.0))
        self.flat = nn.Parameter(_flat.to(device=device, dtype=torch.float32).contiguous())
        self.register_buffer("c_b", torch.ones(3, device=device))
        self.depth_tau_init = depth_tau
        # arm B's global depth weight sigmoid(depth_beta * (depth_tau - z)) (spike/model.py:48-49)
        self.depth_beta = nn.Parameter(torch.tensor(1.0, device=device))
        self.depth_tau = nn.Parameter(torch.tensor(float(depth_tau), device=device))

    @classmethod
    def from_arrays(cls, params, device="cuda"):
        G = int(np.asarray(params["means3d"]).shape[0])
        m = cls(G, device=device, _flat=pack_arrays(params))
        with torch.no_grad():
            for k in ("depth_beta", "depth_tau"):
                if k in params:
                    getattr(m, k).fill_(float(np.asarray(params[k])))
        return m

    @property
    def G(self):
        return self.G_

    def __getattr__(self, name):
        if name in NAMES or name == "w_b_raw":
            return view(self._parameters["flat"], self.G_, name)
        return super().__getattr__(name)

    @torch.no_grad()
    def init_from_points(self, xyz, rgb, seed=0):
        """Start the gaussians from a point cloud (e.g. ``data.load_colmap_points``), as
        spike/model.py:55-79 does: xyz[P,3], rgb[P,3] in [0, 1] (numpy or torch).

        With at least G points, G of them are taken in the order of a random permutation; with
        fewer, every point is kept and the missing G - P are copies of random points, moved by
        Gaussian noise of 1 % of the cloud's bounding-box diagonal.  Every gaussian gets the same
        isotropic log-scale, the log of the median nearest-neighbour distance among up to 4000
        of them (at least 1e-4), and the colour whose DC term renders as the point's rgb.  The
        draws come from a CPU generator seeded with ``seed`` in the reference's order (the
        permutation or the copy indices and noise, then the subset permutation), so a seed
        gives the reference's model; opacities, rotations and SH rest stay as they were."""
        G = self.G_
        gen = torch.Generator().manual_seed(int(seed))
        xyz = torch.as_tensor(xyz, dtype=torch.float32).cpu()
        rgb = torch.as_tensor(rgb, dtype=torch.float32).cpu()
        P = xyz.shape[0]
        if P >= G:
            pick = torch.randperm(P, generator=gen)[:G]
            pts, cols = xyz[pick], rgb[pick]
        else:
            src = torch.randint(0, P, (G - P,), generator=gen)
            diag = (xyz.max(0).values - xyz.min(0).values).norm() * 0.01
            pts = torch.cat([xyz, xyz[src] + torch.randn(G - P, 3, generator=gen) * diag], 0)
            cols = torch.cat([rgb, rgb[src]], 0)
        probe = pts[torch.randperm(G, generator=gen)[:min(G, 4000)]]
        dist = torch.cdist(probe, probe)
        dist.fill_diagonal_(float("inf"))
        nn_dist = dist.min(1).values.median().clamp(min=1e-4)
        dev = self.flat.device
        self.means3d.copy_(pts.to(dev))
        self.log_scales.fill_(float(torch.log(nn_dist)))
        self.color_dc.copy_(((cols - 0.5) / C0).to(dev))
        return self

    def to_arrays(self):
        f = self.flat.detach().cpu()
        out = {n: view(f, self.G_, n).numpy().copy() for n in NAMES}
        out["w_b_raw"] = np.float32(view(f, self.G_, "w_b_raw").item())
        return out


def flat_of(model):
    """The flat parameter tensor of a model: ours directly, or the reference's separate
    parameters concatenated (differentiable, so gradients flow back to them)."""
    if isinstance(model, GaussianModel):
        return model.flat
    G = model.means3d.shape[0]
    dev = model.means3d.device
    rest = getattr(model, "color_rest", None)
    if rest is None:
        rest = torch.zeros(G, 15, 3, device=dev)
    parts = [model.means3d.reshape(-1), model.log_scales.reshape(-1), model.quats.reshape(-1),
             model.opacity_raw.reshape(-1), model.color_dc.reshape(-1), rest.reshape(-1),
             model.w_b_raw.reshape(1)]
    return torch.cat([p.float() for p in parts])


def lr_vector(lr, device):
    """Per-group learning rates of GaussianModel.param_groups (spike/model.py:82-95) in the
    kernel's order: means, log_scales, quats, opacity_raw, color_dc, color_rest, w_b_raw."""
    v = [lr["means"], lr["scales"], lr["quats"], lr["opacity"], lr["color"], lr.get("color_rest", lr["color"] / 20.0),
         lr["wb"]]
    return torch.tensor(v, dtype=torch.float64, device=device)
