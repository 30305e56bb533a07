"""Device-resident, CUDA-graph-captured train step (mirrors spike/train.py:9-41 and the step of
tools/resident_traced.py:667-757).

One ``TrainStep`` owns every buffer of the step for a fixed set of views, so a step allocates
nothing and synchronises nothing with the host:

    step_begin -> project (V views) -> bin + pack -> render forward -> loss forward+gradient
    -> render backward -> slot->gaussian reduction + parameter backward
    [-> NCCL all-reduce of the gradient across ranks] -> Adam (+ SGLD) [-> relocation]

Arms A, B (depth-weighted opacity; the depth group depth_beta/depth_tau gets its own Adam,
spike/model.py:93) and RV (revealage compositing; w_b receives no gradient, so Adam leaves it
where it is, as torch does for a parameter without .grad) train through the same step.

The first step runs eagerly (it also loads the kernels); later steps replay CUDA graphs
captured from the same launches (one graph per step variant: with or without relocation;
with a process group, one graph before and one after the all-reduce).  ``step()`` returns the
device tensor holding the step's mean loss; reading it is the only synchronisation.
"""
import numpy as np
import torch

from . import ops
from ._lib import device_ctx, require_cuda
from .camera import as_camera, pack_cameras
from .model import GaussianModel, flat_of, lr_vector, view

DEFAULT_LR = {"means": 5e-3, "scales": 5e-3, "quats": 1e-3, "opacity": 5e-2, "opacity_sh": 5e-2, "color": 1e-2,
              "wb": 1e-2, "depth": 1e-2}   # spike/train.py:9-12


# Bits of the device status word (tts_read_status): the bounded waits and the table check that
# gave up.  A step that set one of them did not do all of its work.
STATUS_BITS = {
    1: "a bulk-copy wait of the per-tile forward timed out (that tile's pixels were not written)",
    2: "a grid barrier of the relocation kernel timed out (the relocation was abandoned)",
    4: "a peer-exchange wait timed out (a rank's gradient or update never arrived; the waiting "
       "blocks skipped their part of the update)",
    8: "a cached binning table spreads a gaussian over more tiles than its stencil box",
}


def status_message(status):
    """Human-readable description of the bits set in a device status word."""
    parts = [f"{b}: {msg}" for b, msg in STATUS_BITS.items() if status & b]
    unknown = status & ~sum(STATUS_BITS)
    if unknown:
        parts.append(f"unknown bits {unknown:#x}")
    return "; ".join(parts)


def raise_on_status(status, where="training"):
    """Raise RuntimeError naming every bit of a non-zero device status word."""
    if status:
        raise RuntimeError(f"device status {status:#x} during {where}: {status_message(status)}")


def partition_views(n_views, world, rank):
    """The views rank ``rank`` of ``world`` renders: contiguous, as even as possible (ranks beyond
    the number of views get none).  Every rank's gradient carries the 1/n_views scale of the
    reference's mean over cameras (spike/train.py:27), so the sum over ranks is the mean."""
    base, extra = divmod(n_views, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def reduce_across_ranks(grads, loss_sum, group=None):
    """Sum the flat gradient and the per-rank loss sums over the process group (one all-reduce
    each, every rank in the same order)."""
    import torch.distributed as dist
    dist.all_reduce(grads, group=group)
    dist.all_reduce(loss_sum, group=group)


def replica_checksum(flat):
    """Order-independent 64-bit checksum of a parameter buffer's bits (sum of its 32-bit words,
    in int64 so that no addition overflows for buffers below 2^31 words)."""
    return flat.detach().contiguous().view(torch.int32).to(torch.int64).sum().reshape(1)


def replicas_agree(flat, group=None):
    """Whether every rank of ``group`` holds bit-identical parameters: the checksum's min and
    max over the ranks (two all-reduces, every rank in the same order) must coincide.  The
    replicated update keeps replicas equal; this is the periodic check that they are."""
    import torch.distributed as dist
    c = replica_checksum(flat)
    lo, hi = c.clone(), c.clone()
    dist.all_reduce(lo, op=dist.ReduceOp.MIN, group=group)
    dist.all_reduce(hi, op=dist.ReduceOp.MAX, group=group)
    return bool(lo.item() == hi.item())


class TrainStep:
    def __init__(self, model, cameras, gt_images, sh_degree=0, lambda_ssim=0.2, lr=None, K=128, R=1, k=4.0,
                 blur=0.3, near=0.2, noise_lr=0.0, relocate_every=0, dead_thr=0.005, dead_frac=0.0, offset=0.0,
                 lambda_o=0.0, lambda_s=0.0, seed=0, n_views_total=None, process_group=None, use_graph=True,
                 exchange="peer", arm="A"):
        require_cuda()
        if arm not in ("A", "B", "RV"):
            raise NotImplementedError(f"arm {arm!r} is not on the B200 hot path (arms A, B and RV)")
        self.arm = arm
        if not isinstance(model, GaussianModel):
            raise TypeError("TrainStep trains a tt_splat_b200.model.GaussianModel (flat device buffer)")
        self.model = model
        self.flat = model.flat.data
        dev = self.flat.device
        self.dev = dev
        self.G = model.G
        cams = [as_camera(c) for c in cameras]
        self.V = len(cams)
        self.H, self.W = cams[0].H, cams[0].W
        ops.tiles(self.H, self.W)
        self.cams_t = pack_cameras(cams, dev)
        # 8-bit targets (the dataset images' own format) are held and uploaded as uint8 and
        # expanded to x / 255 by the step's first kernel; float targets are used as given
        gts = [torch.as_tensor(g) for g in gt_images]
        self.targets_u8 = None
        if all(g.dtype == torch.uint8 for g in gts):
            self.targets_u8 = torch.stack([g.to(dev) for g in gts]).contiguous()
            self.targets = ops.unit_from_u8(self.targets_u8)
        else:
            self.targets = torch.stack([g.to(dtype=torch.float32).to(dev) for g in gts]).contiguous()
        if tuple(self.targets.shape) != (self.V, self.H, self.W, 3):
            raise ValueError(f"gt images must be [H,W,3] = {(self.H, self.W, 3)} each")
        self.sh_degree, self.lam, self.K, self.R, self.k = int(sh_degree), float(lambda_ssim), int(K), int(R), float(k)
        self.blur, self.near = float(blur), float(near)
        self.noise_lr, self.relocate_every = float(noise_lr), int(relocate_every)
        self.dead_thr, self.dead_frac, self.offset = float(dead_thr), float(dead_frac), float(offset)
        self.lambda_o, self.lambda_s, self.seed = float(lambda_o), float(lambda_s), int(seed)
        self.pg = process_group
        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange must be 'peer' (NVLink peer-memory optimizer step) or 'nccl'")
        self.regions = None
        if self.pg is not None:
            import torch.distributed as dist
            if exchange == "peer" and dist.get_world_size(self.pg) > 1:
                from .peer import PeerRegions
                # parameters and gradients live in the region the peers write into / read from
                if arm == "B":
                    raise NotImplementedError("arm B's depth gradient is reduced by the NCCL exchange: "
                                              "use exchange='nccl'")
                self.regions = PeerRegions(self.flat.numel(), dev, self.pg)
                self.regions.params.copy_(self.flat)
                model.flat.data = self.regions.params
                self.flat = self.regions.params
        self.n_views_total = int(n_views_total or self.V)
        self.grad_scale = 1.0 / self.n_views_total
        self.lr = {**DEFAULT_LR, **(lr or {})}
        self.lr7 = lr_vector(self.lr, dev)
        self.use_graph = use_graph
        G, V, H, W, K = self.G, self.V, self.H, self.W, self.K
        T = (H // 16) * (W // 16)
        S = (2 * self.R + 1) ** 2
        e = lambda *s, dt=torch.float32: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
        self.pj = dict(proj=e(V, G, ops.PROJ_FLOATS), mu2d=e(V, G, 2), keep=e(V, G, dt=torch.uint8),
                       cell_count=torch.zeros(V, T, dtype=torch.int32, device=dev), cell_rank=e(V, G, 2, dt=torch.int32))
        self.bp = dict(idx=e(V, T, K, dt=torch.int32), count=e(V, T, dt=torch.int32), cand=e(V, T, dt=torch.int32),
                       inv=e(V, G, S, dt=torch.int32), slots=e(V, T, K, ops.SLOT_FLOATS))
        self.rf = dict(img=e(V, H, W, 3), den=e(V, H, W))
        if arm == "RV":
            self.rf["aux"] = e(V, H, W, 4)            # (Cavg, R) per pixel for the RV backward
        self.dbt = None
        if arm == "B":
            # the depth group (depth_beta, depth_tau) in one device vector; the model's two
            # parameters become views of it so that they follow the training
            self.dbt = torch.stack([model.depth_beta.detach(), model.depth_tau.detach()]).float().to(dev).contiguous()
            model.depth_beta.data = self.dbt[0]
            model.depth_tau.data = self.dbt[1]
            self.g_dbt, self.m_dbt, self.v_dbt = (torch.zeros(2, device=dev) for _ in range(3))
        self.lo = dict(gimg=e(V, H, W, 3), loss=e(V))   # loss_sum (the step's total) bound below
        self.rb = dict(slot_grads=e(V, T, K, ops.SLOT_GRAD_FLOATS), gwb=e(V, T))
        self.grads = torch.zeros_like(self.flat) if self.regions is None else self.regions.grads
        self.m = torch.zeros_like(self.flat)
        self.v = torch.zeros_like(self.flat)
        self.step_t = torch.zeros(1, dtype=torch.int32, device=dev)
        self.reloc = dict(n_dead=torch.zeros(1, dtype=torch.int32, device=dev), targets=e(G, dt=torch.int32))
        self.ws_bin, self.ws_loss, self.ws_reloc = ops.Workspace(dev), ops.Workspace(dev), ops.Workspace(dev)
        self.ws_bwd = ops.Workspace(dev)
        self.ws_bwd.get(ops.lib().tts_backward_workspace_bytes(G, V))
        self.ws_bin.get(ops.lib().tts_bin_workspace_bytes(G, V, H, W))
        self.ws_loss.get(ops.lib().tts_loss_workspace_bytes(V, H, W))
        self.ws_reloc.get(ops.lib().tts_relocate_workspace_bytes(G) if G >= 2 else 0)
        self.loss_mean = e(1) if self.regions is None else self.regions.loss
        self.lo["loss_sum"] = self.loss_mean   # written by the loss reduction kernel
        self.loss_total = e(1)            # sum over the ranks (peer exchange)
        self.n_moved = torch.zeros(1, dtype=torch.int64, device=dev)
        self.it = 0
        self.graphs = {}
        self.kernels_per_step = None

    # ---- the launches of one step --------------------------------------------------------
    def _fwd_bwd(self):
        G, H, W, R, K = self.G, self.H, self.W, self.R, self.K
        ops.step_begin(self.step_t)
        if self.targets_u8 is not None:
            ops.unit_from_u8(self.targets_u8, out=self.targets)
        ops.project(self.flat, G, self.sh_degree, self.cams_t, H, W, self.blur, self.near, out=self.pj,
                    depth_bt=self.dbt)
        ops.bin_pack(self.pj, G, H, W, R, K, self.k, ws=self.ws_bin, out=self.bp)
        if self.arm == "RV":
            ops.render_fwd_rv(self.bp["slots"], self.bp["count"], H, W, self.model.c_b, out=self.rf)
        else:
            ops.render_fwd(self.bp["slots"], self.bp["count"], H, W, self.flat[59 * G:], self.model.c_b, out=self.rf)
        ops.loss_l1_ssim(self.rf["img"], self.targets, self.lam, self.grad_scale, ws=self.ws_loss, out=self.lo)
        if self.arm == "RV":
            ops.render_bwd_rv(self.bp["slots"], self.bp["count"], H, W, self.model.c_b, self.rf["den"], self.rf["aux"],
                              self.lo["gimg"], out=self.rb)
        else:
            ops.render_bwd(self.bp["slots"], self.bp["count"], H, W, self.model.c_b, self.rf["img"], self.rf["den"],
                           self.lo["gimg"], out=self.rb)
        ops.backward_params(self.flat, G, self.sh_degree, self.cams_t, H, W, R, K, self.bp["inv"],
                            self.rb["slot_grads"], self.rb["gwb"], self.k, self.blur, self.near, self.lambda_o,
                            self.lambda_s, out=self.grads, ws=self.ws_bwd, proj=self.pj["proj"], depth_bt=self.dbt,
                            g_depth_bt=self.g_dbt if self.dbt is not None else None)

    def _update(self, relocate):
        if self.regions is not None:
            # NVLink exchange: signal, (wait) shard reduce + Adam + broadcast (signal), (wait) SGLD;
            # the replicas are bitwise equal afterwards
            ops.peer_signal(self.regions, 0, self.step_t)
            ops.adam_peer(self.regions, self.m, self.v, self.G, self.sh_degree, self.step_t, self.lr7,
                          self.loss_total)
            if relocate and self.noise_lr > 0:
                pass                      # the relocation launch waits for phase 1 and runs SGLD
            elif self.noise_lr > 0:
                ops.peer_sgld(self.regions, self.flat, self.G, self.step_t, self.lr["means"], self.noise_lr,
                              seed=self.seed)
            else:
                ops.peer_wait(self.regions, 1, self.step_t)
        else:
            # a relocating iteration runs its SGLD step inside the relocation launch
            fused = relocate and self.noise_lr > 0
            ops.adam_sgld(self.flat, self.grads, self.m, self.v, self.G, self.sh_degree, self.step_t, self.lr7,
                          noise_lr=0.0 if fused else self.noise_lr, seed=self.seed)
        if self.dbt is not None:
            ops.adam_vec(self.dbt, self.g_dbt, self.m_dbt, self.v_dbt, self.step_t, self.lr["depth"])
        if relocate:
            if self.regions is not None and self.noise_lr > 0:
                ops.peer_sgld_relocate(self.regions, self.flat, self.m, self.v, self.G, self.step_t, self.lr7,
                                       self.noise_lr, dead_thr=self.dead_thr, dead_frac=self.dead_frac,
                                       offset=self.offset, seed=self.seed, ws=self.ws_reloc, out=self.reloc)
            elif self.noise_lr > 0:
                ops.sgld_relocate(self.flat, self.m, self.v, self.G, self.step_t, self.lr7, self.noise_lr,
                                  dead_thr=self.dead_thr, dead_frac=self.dead_frac, offset=self.offset,
                                  seed=self.seed, ws=self.ws_reloc, out=self.reloc)
            else:
                ops.relocate(self.flat, self.m, self.v, self.G, self.step_t, self.dead_thr, self.dead_frac,
                             self.offset, seed=self.seed, ws=self.ws_reloc, out=self.reloc)
            self.n_moved.add_(self.reloc["n_dead"])

    def _allreduce(self):
        reduce_across_ranks(self.grads, self.loss_mean, self.pg)
        if self.dbt is not None:
            import torch.distributed as dist
            dist.all_reduce(self.g_dbt, group=self.pg)

    def _run(self, relocate):
        if self.pg is None or self.regions is not None:
            self._fwd_bwd()
            self._update(relocate)
        else:
            self._fwd_bwd()
            self._allreduce()
            self._update(relocate)

    def _graph_run(self, relocate):
        if self.pg is None or self.regions is not None:
            key = ("all", relocate)
            if key not in self.graphs:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._fwd_bwd()
                    self._update(relocate)
                self.graphs[key] = g
            self.graphs[key].replay()
        else:
            if "fb" not in self.graphs:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._fwd_bwd()
                self.graphs["fb"] = g
            key = ("up", relocate)
            if key not in self.graphs:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._update(relocate)
                self.graphs[key] = g
            self.graphs["fb"].replay()
            self._allreduce()
            self.graphs[key].replay()

    def phase_times(self, steps=20):
        """Device time of the two halves of a step on this rank, from separately captured graphs:
        (forward/backward chain ms, exchange + update ms).  With several ranks the second half
        includes the wait for the slowest rank's first half.  Runs `steps` training steps."""
        relocate = bool(self.relocate_every) and self.G >= 2
        if self.pg is not None and self.regions is None:
            raise RuntimeError("phase_times needs the single-process or peer-exchange step")
        if "fb" not in self.graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._fwd_bwd()
            self.graphs["fb"] = g
        key = ("up", relocate)
        if key not in self.graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._update(relocate)
            self.graphs[key] = g
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        fb = up = 0.0
        for _ in range(steps):
            # a device-side spin ahead of the two replays lets the host enqueue both before the
            # GPU reaches them, so the halves are device time, not host graph-launch latency
            torch.cuda._sleep(2_000_000)
            ev[0].record()
            self.graphs["fb"].replay()
            ev[1].record()
            self.graphs[key].replay()
            ev[2].record()
            torch.cuda.synchronize()
            fb += ev[0].elapsed_time(ev[1])
            up += ev[1].elapsed_time(ev[2])
            self.it += 1
        return fb / steps, up / steps

    def launches(self, relocate):
        """Kernels of this library launched by one step (memsets and torch ops excluded):
        step_begin 1, [8-bit target expansion 1], project 1, bin_pack 4, render_fwd 1, loss 3, render_bwd 1,
        backward_params 3, then Adam (+ SGLD) or the peer step (2 barriers + Adam + SGLD), and
        the relocation kernel (on one GPU it also runs the SGLD step of a relocating iteration)."""
        n = 14 + (1 if self.targets_u8 is not None else 0)
        if self.regions is not None:
            n += 2 + (0 if relocate and self.noise_lr > 0 else 1)   # signal, Adam, SGLD or wait
        else:
            n += 1 + (1 if self.noise_lr > 0 and not relocate else 0)
        if self.dbt is not None:
            n += 1                                       # Adam of the depth group (arm B)
        if relocate:
            n += 1
        return n

    def step(self):
        """One training iteration (spike/mcmc.py:97-111 order); returns the device loss tensor."""
        it = self.it
        relocate = bool(self.relocate_every) and it > 0 and it % self.relocate_every == 0 and self.G >= 2
        self.kernels_per_step = self.launches(relocate)
        with torch.cuda.device(self.dev):
            if self.use_graph and it > 0:
                self._graph_run(relocate)
            else:
                self._run(relocate)
        self.it += 1
        return (self.loss_mean if self.regions is None else self.loss_total).view(())

    def mean_loss_value(self):
        """Mean photometric loss of the last step (+ the MCMC regulariser when enabled); syncs."""
        total = float((self.loss_mean if self.regions is None else self.loss_total).item()) / self.n_views_total
        if self.lambda_o or self.lambda_s:
            o = torch.sigmoid(view(self.flat, self.G, "opacity_raw"))
            s = torch.exp(view(self.flat, self.G, "log_scales"))
            total += self.lambda_o * float(o.mean()) + self.lambda_s * float(s.mean())
        return total

    def check_status(self):
        """Read and clear the device status word (synchronises); raise RuntimeError naming the
        bits when a bounded wait gave up since the last check, i.e. when a step skipped work."""
        with device_ctx(self.dev):
            raise_on_status(ops.read_status(), f"the steps up to iteration {self.it}")

    def check_replicas(self):
        """Raise if a bounded wait gave up (``check_status``) or the ranks' parameter replicas
        have diverged (the replica check is a no-op without a process group)."""
        self.check_status()
        if self.pg is None:
            return
        if not replicas_agree(self.flat, self.pg):
            raise RuntimeError(f"parameter replicas differ across ranks after step {self.it}")

    def release(self):
        """Drop the captured graphs and, with the peer exchange, hand the model a private copy of
        its parameters and free the shared regions (call before destroying a process group;
        every rank calls it)."""
        self.graphs.clear()
        if self.regions is not None:
            own = self.flat.clone()
            self.model.flat.data = own
            self.flat = own
            self.regions.close()
            self.regions = None


def fit(model, cameras, gt_images, arm="A", iters=800, lambda_ssim=0.2, lr=None, k=4.0, blur_eps=0.3, near=0.2,
        log_every=0, sh_degree=0, K=128, R=1):
    """spike/train.py:15-33 on the B200 path: returns the per-iteration mean loss history."""
    st = TrainStep(model, cameras, gt_images, sh_degree=sh_degree, lambda_ssim=lambda_ssim, lr=lr, K=K, R=R, k=k,
                   blur=blur_eps, near=near, arm=arm)
    hist = []
    for it in range(iters):
        hist.append(st.step().clone())
        if log_every and (it % log_every == 0 or it == iters - 1):
            print(f"    iter {it:4d}  loss {float(hist[-1]) / st.V:.5f}")
    st.check_status()
    return (torch.stack(hist) / st.V).cpu().tolist() if hist else []


@torch.no_grad()
def eval_psnr(model, cameras, gt_images, arm="A", **kw):
    """spike/train.py:36-41."""
    from .metrics import psnr
    from .render import render
    vals = [float(psnr(render(model, cam, arm, **kw), torch.as_tensor(gt).to(model.flat.device)))
            for cam, gt in zip(cameras, gt_images)]
    return sum(vals) / len(vals)
