"""Oracle (test and baseline infrastructure only): the whole train step of the CPU restatement,
with the batch's views spread over worker processes.

The reference trains on a batch of views whose per-view forward + loss + backward are independent
(``spike/mcmc.py:90-114``: mean of the per-view losses, one optimizer step).  ``CpuStep`` runs
those per-view passes in parallel, one worker process per view up to the host's cores and
memory, each numpy process given the host's cores divided by the workers as BLAS threads, then
sums the per-view gradients in view order and applies Adam, SGLD noise and relocation in the calling process.  (Splitting a view's
tiles over threads of one worker measured slower than one thread: the page faults of the large
per-tile temporaries contend inside a process.)  It is timed as the CPU baseline of the
benchmark; it is never part of the product.

Workers are started with ``spawn`` so that a caller that already holds a CUDA context can use it.
The scene reaches them through a temporary file, so the start-up message each worker reads from
its pipe stays small: a worker that dies then makes the step raise (``BrokenProcessPool``)
instead of leaving the parent blocked on a pipe nobody drains.
"""
import multiprocessing as mp
import os
import pickle
import tempfile
from concurrent.futures import ProcessPoolExecutor

import numpy as np

from . import loss as loss_mod
from . import optim
from . import pipeline

LR = {"means": 1.6e-4, "scales": 5e-3, "quats": 1e-3, "opacity": 5e-2, "color": 1e-2, "wb": 1e-2}
VIEW_PEAK_BYTES = 3.0e9      # measured peak of one config-2 view (2.45 GB) with margin
_BLAS_VARS = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")

_W = {}


def _init(scene_path):
    with open(scene_path, "rb") as f:
        _W.update(pickle.load(f))


def _view(v):
    """Forward + L1/SSIM loss + backward of view ``v`` (the loss averaged over the batch)."""
    p, d = _W["params"], _W["sh_degree"]
    fw = pipeline.render_view(p, d, _W["cams"][v], K=_W["K"])
    loss, _, _, gimg = loss_mod.loss_and_grad(fw["img"], _W["targets"][v], 0.2)
    g = pipeline.backward_view(fw, (gimg / _W["n_views"]).astype(np.float32), p, d)
    return v, float(loss), g


def host_cores():
    """Cores this process may run on."""
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def host_workers(n_views, per_view_bytes=VIEW_PEAK_BYTES):
    """Worker count: one per view, bounded by the cores and by 60% of the available memory."""
    cores = host_cores()
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except ImportError:
        avail = per_view_bytes
    return max(1, min(n_views, cores, int(0.6 * avail // per_view_bytes)))


class CpuStep:
    """One train step of the oracle over all views of a scene (``synthetic.config2()`` form)."""

    def __init__(self, scene, workers=None, seed=0):
        self.p = scene["params"]
        self.sh_degree = scene.get("sh_degree", 3)
        self.n_views = len(scene["cams"])
        self.workers = workers or host_workers(self.n_views)
        self.rng = np.random.default_rng(seed)
        fd, self.scene_path = tempfile.mkstemp(prefix="ttsplat_scene_", suffix=".pkl")
        saved = {k: os.environ.get(k) for k in _BLAS_VARS}
        try:
            with os.fdopen(fd, "wb") as f:
                pickle.dump(dict(params=self.p, sh_degree=self.sh_degree, cams=scene["cams"],
                                 targets=scene["targets"], K=scene.get("K", 128), n_views=self.n_views),
                            f, protocol=pickle.HIGHEST_PROTOCOL)
            # the host's cores split over the workers (one BLAS thread each when there are no more
            # cores than views)
            self.threads_per_worker = max(1, host_cores() // self.workers)
            for k in _BLAS_VARS:
                os.environ[k] = str(self.threads_per_worker)
            self.pool = ProcessPoolExecutor(self.workers, mp_context=mp.get_context("spawn"), initializer=_init,
                                            initargs=(self.scene_path,))
        except BaseException:
            os.unlink(self.scene_path)
            raise
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v

    def loss_and_grads(self, lambda_o=0.01, lambda_s=0.01):
        """Mean photometric loss over the views and the summed per-view gradients (view order),
        plus the MCMC regulariser's gradient (spike/mcmc.py:102, reg_loss :18-22)."""
        res = sorted(self.pool.map(_view, range(self.n_views)), key=lambda r: r[0])
        g = {k: np.array(res[0][2][k], copy=True) if k != "w_b_raw" else res[0][2][k] for k in res[0][2]}
        for _, _, gv in res[1:]:
            for k in g:
                g[k] = g[k] + gv[k]
        if lambda_o or lambda_s:
            gop, gls = optim.reg_loss_grads(self.p["opacity_raw"], self.p["log_scales"], lambda_o, lambda_s)
            g["opacity_raw"] = g["opacity_raw"] + gop
            g["log_scales"] = g["log_scales"] + gls
        return sum(r[1] for r in res) / self.n_views, g

    def step(self):
        """Run one step; returns (photometric loss, updated parameter copy)."""
        loss, g = self.loss_and_grads()
        q = pipeline.copy_params(self.p)
        pipeline.adam_step(q, g, {}, 1, LR, self.sh_degree)
        G = self.p["means3d"].shape[0]
        q["means3d"] = optim.sgld_noise(q["means3d"], q["log_scales"], q["quats"], q["opacity_raw"],
                                        self.rng.standard_normal((G, 3)), LR["means"]).astype(np.float32)
        o = 1 / (1 + np.exp(-q["opacity_raw"].astype(np.float64)))
        thr = optim.quantile_threshold(o, 0.01)
        n_dead = int((o < thr).sum())
        alive = np.nonzero(o >= thr)[0]
        tgts = alive[self.rng.choice(alive.size, n_dead, p=o[alive] / o[alive].sum())]
        optim.relocate(q, thr, tgts)
        return loss, q

    def close(self):
        try:
            self.pool.shutdown(wait=True, cancel_futures=True)
        finally:
            if os.path.exists(self.scene_path):
                os.unlink(self.scene_path)

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
