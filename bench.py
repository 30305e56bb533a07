"""Benchmark of the headline workload: the device-resident, graph-captured 3DGS train step.

Workload (benchmark config 2): G = 100,000 gaussians, SH degree 3, a batch of 8 cameras on a
radius-4 ring (1264x832, 16x16 tiles, K = 128, R = 1), 0.8*L1 + 0.2*(1-SSIM) loss with the
11x11 window, fused Adam (lr 1.6e-4 on means, beta 0.9/0.999), MCMC SGLD noise (noise_lr 5e5)
and relocation of the 1% lowest-opacity gaussians every step, plus the MCMC regulariser.
Views are split over the ranks; the gradient exchange and the sharded Adam step run over NVLink
peer memory inside the step's CUDA graph (no library collective on the data path).
One step = the whole 8-view batch, so ``value`` (steps/s) is a whole-job number and the
scaling is strong (fixed total work).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the CPU restatement of the reference path (the oracle port; the
reference itself is Python and cannot travel to the GPU box): whole 8-view steps, the views'
forward + loss + backward spread over worker processes on the host cores, for at most 90 s.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import __graft_entry__  # noqa: E402

CONFIG = dict(workload="config2: train step, G=100k, 8 views 1264x832, K=128, SH3, MCMC", G=100000, views=8,
              H=832, W=1264, K=128, R=1, sh_degree=3,
              l2="inputs larger than L2: the per-step working set (~1 GB: targets, images, slot rows, SSIM maps) "
                 "exceeds the 126 MB L2")
METRIC = "train steps/s (G=100k, 8-view batch 1264x832, 1/2/4/8 B200)"
PEAKS_FILE = os.path.join(REPO, "MEASURED_PEAKS.json")
REF_BUDGET_S = 90.0   # wall-clock budget of the CPU reference arm's timed samples
CPU_SAMPLE = ("median of whole steps after one warm-up step: the 8 views' forward+loss+backward on "
              "{workers} worker processes (one per view, {threads} BLAS thread(s) each), gradients summed in view "
              "order, then Adam, SGLD and 1% relocation over all 100k gaussians; numpy oracle")


def load_peaks():
    try:
        with open(PEAKS_FILE) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "sm_max_mhz": 1965.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                for line in out.stdout.strip().splitlines():
                    self.samples.append([x.strip() for x in line.split(",")])
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if len(s) > 5 + i and "Active" in s[5 + i]
                          and "Not" not in s[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ----------------------------------------------------------------------------------------------
def run_reference(args, rank, world):
    """The CPU restatement of the reference train step (rank 0 only): every step runs all views'
    forward + loss + backward over worker processes (one BLAS thread each, one view per worker up
    to the host's cores and memory), sums the gradients and applies Adam, SGLD and relocation."""
    if rank != 0:
        return
    from oracle.step import CpuStep, host_cores
    pkg = __graft_entry__.load_package()
    with CpuStep(pkg.synthetic.config2()) as cs:
        # one step takes seconds: one warm-up step (it also starts the workers), then timed
        # steps until the requested count or a 90-s budget (at least three; the median is kept)
        warm = 1
        cs.step()
        times = []
        t_start = time.perf_counter()
        while len(times) < max(args.steps, 3) and (len(times) < 3 or time.perf_counter() - t_start < REF_BUDGET_S):
            t0 = time.perf_counter()
            cs.step()
            times.append(time.perf_counter() - t0)
        workers, threads = cs.workers, cs.threads_per_worker
    step_s = float(np.median(times))
    line = {"impl": "reference", "metric": METRIC, "value": 1.0 / step_s, "unit": "steps/s", "n_gpus": world,
            "steps": len(times), "warmup": warm, "steps_requested": args.steps, "warmup_requested": args.warmup,
            "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, config 2 shapes)",
            "config": {k: v for k, v in CONFIG.items()},
            "cpu_baseline": {"value": 1.0 / step_s, "unit": "steps/s", "cores": workers * threads, "kind": "port",
                             "host_cores": host_cores(),
                             "note": "numpy port of the reference path: one worker process per view, the host's "
                                     "cores divided over them as BLAS threads",
                             "sample": CPU_SAMPLE.format(workers=workers, threads=threads)},
            "e2e": {"value": 1.0 / step_s, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------------
def stage_times(st, torch, reps=3):
    """Per-stage device times of one eager step (CUDA events on the launching stream, the stages
    queued behind a device-side spin so that host launch latency is excluded)."""
    from tt_splat_b200 import ops
    names = ["targets_u8", "project", "bin_pack", "render_fwd", "loss", "render_bwd", "backward_params", "adam", "sgld",
             "relocate"]
    acc = {n: [] for n in names}
    G, H, W, R, K = st.G, st.H, st.W, st.R, st.K
    for _ in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
        # a device-side spin ahead of the stages lets the host enqueue them all before the GPU
        # reaches them, so the event deltas are device time, not host launch latency
        torch.cuda._sleep(4_000_000)
        ev[0].record()
        ops.step_begin(st.step_t)
        if st.targets_u8 is not None:
            ops.unit_from_u8(st.targets_u8, out=st.targets)
        ev[1].record()
        ops.project(st.flat, G, st.sh_degree, st.cams_t, H, W, st.blur, st.near, out=st.pj)
        ev[2].record()
        ops.bin_pack(st.pj, G, H, W, R, K, st.k, ws=st.ws_bin, out=st.bp)
        ev[3].record()
        ops.render_fwd(st.bp["slots"], st.bp["count"], H, W, st.flat[59 * G:], st.model.c_b, out=st.rf)
        ev[4].record()
        ops.loss_l1_ssim(st.rf["img"], st.targets, st.lam, st.grad_scale, ws=st.ws_loss, out=st.lo)
        ev[5].record()
        ops.render_bwd(st.bp["slots"], st.bp["count"], H, W, st.model.c_b, st.rf["img"], st.rf["den"],
                       st.lo["gimg"], out=st.rb)
        ev[6].record()
        ops.backward_params(st.flat, G, st.sh_degree, st.cams_t, H, W, R, K, st.bp["inv"], st.rb["slot_grads"],
                            st.rb["gwb"], st.k, st.blur, st.near, st.lambda_o, st.lambda_s, out=st.grads, ws=st.ws_bwd,
                            proj=st.pj["proj"])
        ev[7].record()
        ops.adam_sgld(st.flat, st.grads, st.m, st.v, G, st.sh_degree, st.step_t, st.lr7, noise_lr=0.0)
        ev[8].record()
        ops.sgld(st.flat, G, st.step_t, st.lr["means"], st.noise_lr, seed=st.seed)
        ev[9].record()
        ops.relocate(st.flat, st.m, st.v, G, st.step_t, st.dead_thr, st.dead_frac, st.offset, seed=st.seed,
                     ws=st.ws_reloc, out=st.reloc)
        ev[10].record()
        torch.cuda.synchronize()
        for i, n in enumerate(names):
            acc[n].append(ev[i].elapsed_time(ev[i + 1]))
    return {n: float(np.median(v)) for n, v in acc.items()}


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    pkg = __graft_entry__.load_package()
    from tt_splat_b200 import camera, model, ops, train
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    sc = pkg.synthetic.config2(G=CONFIG["G"], n_views=max(CONFIG["views"], 1))
    V = CONFIG["views"]
    mine = train.partition_views(V, world, rank)
    if not mine:
        raise SystemExit(f"rank {rank}: more ranks than views ({V})")
    cams = [camera.Camera.from_dict(sc["cams"][i]) for i in mine]
    # the targets are 8-bit images: uploaded as uint8, expanded to x / 255 on the device each step
    targets_host = torch.from_numpy(np.stack([sc["targets_u8"][i] for i in mine])).pin_memory()
    m = model.GaussianModel.from_arrays(sc["params"], device=dev)
    pg = dist.group.WORLD if world > 1 else None
    st = train.TrainStep(m, cams, list(targets_host), sh_degree=3, lr={"means": 1.6e-4}, K=CONFIG["K"], R=CONFIG["R"],
                         noise_lr=5e5, relocate_every=1, dead_frac=0.01, offset=0.005, lambda_o=0.01, lambda_s=0.01,
                         seed=1234, n_views_total=V, process_group=pg, exchange=args.exchange)

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up: the first step runs eagerly (loads kernels), the next capture the graphs
    for _ in range(max(args.warmup, 3)):
        st.step()
    torch.cuda.synchronize()
    # per-stage device times on rank 0; its parameters, moments and step counter are restored
    # afterwards so that the ranks stay in lockstep (same step, bitwise-equal replicas)
    stages = None
    if rank == 0:
        snap = [t.clone() for t in (st.flat, st.m, st.v, st.step_t)]
        stages = stage_times(st, torch)
        for t, c in zip((st.flat, st.m, st.v, st.step_t), snap):
            t.copy_(c)
        del snap
    torch.cuda.synchronize()
    fp32_peak = ops.fp32_peak_tflops() if rank == 0 else None
    ops.read_status()          # clear the device status word before the timed region
    barrier()
    # Every leg below starts from this state.  SGLD at noise_lr 5e5 on random-noise targets
    # carries near-transparent gaussians far from the scene (some towards the camera planes,
    # where the fp32 conic inverse of spike/geometry.py overflows), and a model trained on that
    # workload for many hundreds of steps produces non-finite pixels, which would change the
    # work later legs measure.
    start = [t.clone() for t in (st.flat, st.m, st.v, st.step_t)]

    def restore():
        for t, c in zip((st.flat, st.m, st.v, st.step_t), start):
            t.copy_(c)
        torch.cuda.synchronize()
        barrier()

    # ---- device-timed region: graph replays, inputs resident ---------------------------------
    with ClockSampler(local_rank) as clk:
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            st.step()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    steps_per_s = args.steps / (ms / 1e3)
    finite = bool(torch.isfinite(st.flat).all().item())
    restore()

    # ---- end to end through the public API: pinned H2D of the step's targets, D2H of the loss
    # Every step uploads its 8 target images (8-bit, 25 MB) from pinned host memory and reads its
    # loss back to the host.  The upload of step i+1 runs on a copy stream while step i computes
    # (double-buffered staging), the way a training loop streams its next batch; both sit inside
    # the timed region.
    h2d = targets_host.numel() * targets_host.element_size()
    if args.skip_e2e:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": steps_per_s, "unit": "steps/s", "config": CONFIG,
                              "stage_ms": stages}), flush=True)
        st.release()
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    copy_stream = torch.cuda.Stream()
    staging = [torch.empty_like(st.targets_u8) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    main = torch.cuda.current_stream()
    barrier()
    torch.cuda.synchronize()
    e0.record()
    with torch.cuda.stream(copy_stream):
        staging[0].copy_(targets_host, non_blocking=True)
        copied[0].record(copy_stream)
    # each step's loss is copied to pinned host memory without blocking and read on the host one
    # step later (the way a training loop logs), so the GPU always has the next step queued
    loss_pinned = torch.zeros(2, dtype=torch.float32).pin_memory()
    loss_ready = [torch.cuda.Event() for _ in range(2)]
    losses_host = []
    for i in range(args.steps):
        b = i % 2
        if i + 1 < args.steps:
            nb = (i + 1) % 2
            with torch.cuda.stream(copy_stream):
                if i >= 1:
                    copy_stream.wait_event(consumed[nb])
                staging[nb].copy_(targets_host, non_blocking=True)
                copied[nb].record(copy_stream)
        main.wait_event(copied[b])
        st.targets_u8.copy_(staging[b], non_blocking=True)
        consumed[b].record(main)
        loss_pinned[b:b + 1].copy_(st.step().view(1), non_blocking=True)
        loss_ready[b].record(main)
        if i >= 1:
            loss_ready[1 - b].synchronize()
            losses_host.append(float(loss_pinned[1 - b]))
    loss_ready[(args.steps - 1) % 2].synchronize()
    losses_host.append(float(loss_pinned[(args.steps - 1) % 2]))
    e1.record()
    torch.cuda.synchronize()
    assert len(losses_host) == args.steps
    barrier()
    ms_e2e = e0.elapsed_time(e1)
    t = torch.tensor([ms_e2e], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_e2e = float(t.item())
    # bounded device waits that gave up during the timed steps (0 = none), max over ranks
    status = torch.tensor([ops.read_status()], device=dev)
    if world > 1:
        dist.all_reduce(status, op=dist.ReduceOp.MAX)
    status = int(status.item())
    # per-rank halves of the step (outside the timed region): the forward/backward chain of this
    # rank's views, and the exchange + update, which waits for the slowest rank
    phases = None
    if world > 1 and st.regions is not None:
        fb_ms, up_ms = st.phase_times(20)
        pt = torch.tensor([fb_ms, up_ms], device=dev)
        allp = [torch.zeros_like(pt) for _ in range(world)]
        dist.all_gather(allp, pt)
        phases = {"fwd_bwd_ms": [round(float(x[0]), 4) for x in allp],
                  "exchange_update_ms": [round(float(x[1]), 4) for x in allp]}
    # the replicated update must leave every rank with the same parameter bits (outside timing)
    replicas_ok = True
    if world > 1:
        from tt_splat_b200.train import replicas_agree
        replicas_ok = replicas_agree(st.flat, pg)

    # ---- render MPix/s: forward of the 8-view batch (project + bin + render), device-timed ----
    restore()
    rend_ms = None
    if rank == 0:
        pj, bp, rf = st.pj, st.bp, st.rf
        for _ in range(3):
            ops.project(st.flat, st.G, 3, st.cams_t, st.H, st.W, out=pj)
            ops.bin_pack(pj, st.G, st.H, st.W, st.R, st.K, ws=st.ws_bin, out=bp)
            ops.render_fwd(bp["slots"], bp["count"], st.H, st.W, st.flat[59 * st.G:], st.model.c_b, out=rf)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(10):
            ops.project(st.flat, st.G, 3, st.cams_t, st.H, st.W, out=pj)
            ops.bin_pack(pj, st.G, st.H, st.W, st.R, st.K, ws=st.ws_bin, out=bp)
            ops.render_fwd(bp["slots"], bp["count"], st.H, st.W, st.flat[59 * st.G:], st.model.c_b, out=rf)
        e1.record()
        torch.cuda.synchronize()
        rend_ms = e0.elapsed_time(e1) / 10

    if rank == 0:
        peaks, peak_src = load_peaks()
        counts = st.bp["count"].long()
        pairs = int(counts.sum().item()) * 256
        # dominant kernel: the fused per-tile backward, FP32-pipe bound (44 flops per valid pair)
        bwd_ms = stages["render_bwd"]
        clk_s = clk.summary()
        sm_mhz = clk_s["sm_mhz"] or peaks.get("sm_max_mhz", 1965.0)
        fp32_nominal = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12     # TFLOP/s at the sampled SM clock
        achieved = 44.0 * pairs / (bwd_ms * 1e-3) / 1e12
        adam_gbs = 28.0 * (59 * st.G + 1) / (stages["adam"] * 1e-3) / 1e9
        adam_dram_gbs = ADAM_DRAM / (stages["adam"] * 1e-3) / 1e9
        launches = st.kernels_per_step or 0
        line = {
            "metric": METRIC, "value": steps_per_s, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, config 2 shapes; random-init model)",
            "config": dict(CONFIG), "views_per_rank": len(mine),
            "parallelism": (f"view-split x{world} + NVLink peer optimizer step" if st.regions is not None
                            else f"view-split x{world}" + (" + NCCL allreduce" if world > 1 else "")),
            "render_mpix_s": (V * CONFIG["H"] * CONFIG["W"] / 1e6) / (rend_ms / 1e3) if rend_ms and world == 1 else None,
            "roofline": {"bound": "fp32", "kernel": "render_bwd", "achieved": achieved, "peak": fp32_peak,
                         "unit": "TFLOP/s", "frac": achieved / fp32_peak,
                         "traffic": RENDER_BWD_DRAM_PER_VIEW * V if CONFIG["G"] == 100000 else None,
                         "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                                         "4-view capture scaled by views per launch)",
                         "traffic_source": TRAFFIC_SOURCE,
                         "peak_source": "measured in this run: packed fma.rn.f32x2 probe kernel (tts_fma_probe, best "
                                        "of 5 launches); MEASURED_PEAKS.json has no FP32 figure",
                         "peak_nominal": fp32_nominal,
                         "work": f"44 flops x {pairs} valid (pixel, slot) pairs per launch"},
            "roofline_hbm": {"bound": "hbm", "kernel": "adam", "achieved": adam_gbs, "peak": peaks.get("hbm_gbs"),
                             "unit": "GB/s", "frac": adam_gbs / peaks.get("hbm_gbs", 6538.0),
                             "traffic": ADAM_DRAM if CONFIG["G"] == 100000 else None,
                             "traffic_source": TRAFFIC_SOURCE,
                             "dram_achieved": adam_dram_gbs, "dram_frac": adam_dram_gbs / peaks.get("hbm_gbs", 6538.0),
                             "work": f"28 B x {59 * st.G + 1} parameter elements per launch (read p,g,m,v; write p,m,v); "
                                     "dram_* use the ncu DRAM bytes (part of p, m, v stays in L2)"},
            "stage_ms": stages, "clocks": clk_s, "replicas_agree": replicas_ok, "device_status": status, "params_finite_after_timed_steps": finite, "rank_phases": phases,
            "e2e": {"value": args.steps / (ms_e2e / 1e3), "unit": "steps/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 4},
            "gpu_launches": launches * args.steps,
            "peaks": {"hbm_gbs": peaks.get("hbm_gbs"), "source": peak_src},
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample()
        print(json.dumps(line), flush=True)
    st.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_config(args, rank, world, local_rank, cid):
    """Benchmark configs 1, 3 and 4 (extra lines; the headline is config 2).

    config 1: G = 10k in 8 clusters, SH 3, one 800x800 view, K = 128: forward + L1 + backward
              with fp32 slot rows (the line's value), and the bf16-operand forward alone
              (fwd_bf16_*); every rank runs the same view (replicas).
    config 3: G = 1M clustered, 1920x1072 (1080 cropped to whole tiles), K = 256, fp32; each rank
              renders one view forward + backward (weak scaling); reports candidate overflow.
    config 4: G = 3M, 64 views 1264x832 on a seeded spiral, K = 128, forward only from compact
              bf16 slot rows; views partitioned over the ranks with no collective (strong
              scaling); frames/s, MPix/s.
    """
    import torch
    import torch.distributed as dist
    pkg = __graft_entry__.load_package()
    from tt_splat_b200 import camera, ops, train
    from tt_splat_b200.model import pack_arrays
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if cid == 1:
        sc = pkg.synthetic.config1()
        mine = [0]                               # one view: every rank runs a replica
    elif cid == 3:
        sc = pkg.synthetic.config3(n_views=max(world, 1))
        mine = [rank]
    else:
        sc = pkg.synthetic.config4()
        mine = train.partition_views(len(sc["cams"]), world, rank)
    p = sc["params"]
    G, K, sh = p["means3d"].shape[0], sc["K"], sc["sh_degree"]
    H, W = sc["cams"][0]["H"], sc["cams"][0]["W"]
    flat = pack_arrays(p).to(dev)
    c_b = torch.ones(3, device=dev)
    chunk = 8                                   # views per launch (bounds the per-view buffers)
    groups = [mine[i:i + chunk] for i in range(0, len(mine), chunk)]
    cams_t = [camera.pack_cameras([camera.Camera.from_dict(sc["cams"][i]) for i in gv], dev) for gv in groups]
    ws = ops.Workspace(dev)
    state = {"wsl": ops.Workspace(dev), "wsb": ops.Workspace(dev)}
    # the loss target stays resident: config 1's seeded target image, config 3's seeded uniform
    # image (one view of H x W x 3)
    if cid == 1:
        state["tg"] = torch.from_numpy(sc["targets"][0]).to(dev)[None].contiguous()
    elif cid == 3:
        state["tg"] = torch.rand((len(groups[0]), H, W, 3), device=dev, generator=torch.Generator(dev).manual_seed(5))

    def once(fwd_bf16=False, marks=None):
        # marks: a list that receives (stage, recorded CUDA event) pairs for the first view group
        def tick(name):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((name, ev))

        for gi, ct in enumerate(cams_t):
            if marks is not None and gi > 0:
                break
            tick("start")
            pj = ops.project(flat, G, sh, ct, H, W, out=state.get("pj"))
            state["pj"] = pj
            tick("project")
            bf16 = cid == 4 or fwd_bf16
            key = "bp16" if bf16 else "bp"
            bp = ops.bin_pack(pj, G, H, W, 1, K, ws=ws, out=state.get(key), with_inv=cid in (1, 3) and not bf16,
                              bf16=bf16)
            state[key] = bp
            tick("bin_pack")
            rf = ops.render_fwd(bp["slots"], bp["count"], H, W, flat[59 * G:], c_b, out=state.get("rf"), bf16=bf16)
            state["rf"] = rf
            tick("render_fwd")
            if cid in (1, 3) and not fwd_bf16:
                tg = state["tg"]
                # config 1: the L1 loss of its reference run (tools/m4_train_binned.py:238-248);
                # config 3: the train step's L1 + SSIM
                lo = ops.loss_l1_ssim(rf["img"], tg, 0.0 if cid == 1 else 0.2, 1.0, ws=state["wsl"],
                                      out=state.get("lo"))
                state["lo"] = lo
                tick("loss")
                rb = ops.render_bwd(bp["slots"], bp["count"], H, W, c_b, rf["img"], rf["den"], lo["gimg"],
                                    out=state.get("rb"))
                state["rb"] = rb
                tick("render_bwd")
                state["grads"] = ops.backward_params(flat, G, sh, ct, H, W, 1, K, bp["inv"], rb["slot_grads"],
                                                     rb["gwb"], out=state.get("grads"), ws=state["wsb"],
                                                     proj=pj["proj"])
                tick("backward_params")

    for _ in range(max(args.warmup, 3)):
        once()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, min(args.steps, 200 if cid == 1 else 50 if cid == 3 else 10))
    e0.record()
    for _ in range(steps):
        once()
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    fwd16_ms = None
    if cid == 1:
        # the bf16-operand forward alone (project + bin with compact rows + render)
        for _ in range(3):
            once(fwd_bf16=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            once(fwd_bf16=True)
        e1.record()
        torch.cuda.synchronize()
        fwd16_ms = e0.elapsed_time(e1) / steps
    # per-stage device time of one launch of the first view group (CUDA events between the
    # stages, mean of five passes)
    stage_ms = {}
    for _ in range(5):
        marks = []
        once(marks=marks)
        torch.cuda.synchronize()
        for (_, a), (name, b) in zip(marks, marks[1:]):
            stage_ms[name] = stage_ms.get(name, 0.0) + a.elapsed_time(b) / 5
    if cid == 3:
        cand = state["bp"]["cand"].reshape(-1).long()
        over = torch.clamp(cand - K, min=0)
        extra = {"overflow_tiles": int((over > 0).sum()), "overflow_total": int(over.sum()),
                 "max_candidates": int(cand.max())}
    else:
        extra = {}
    n_views_job = world if cid in (1, 3) else len(sc["cams"])
    if cid == 1:
        extra = {"overflow_tiles": int((state["bp"]["cand"] > K).sum()),
                 "fwd_bf16_ms": fwd16_ms, "fwd_bf16_mpix_s": H * W / 1e6 / (fwd16_ms / 1e3),
                 "loss": "L1 (the reference's config-1 run)", "replicas": "every rank runs the single view"}
    if rank == 0:
        metric = {1: "fwd+bwd views/s (config 1)", 3: "fwd+bwd views/s (config 3)", 4: "render frames/s (config 4)"}[cid]
        line = {"metric": metric,
                "value": n_views_job / (ms / 1e3), "unit": "frames/s" if cid == 4 else "views/s",
                "n_gpus": world, "steps": steps, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong" if cid == 4 else "weak",
                "dtype": "bf16 slot rows, f32 accumulate" if cid == 4 else "f32", "data": "synthetic (seeded)",
                "mpix_s": n_views_job * H * W / 1e6 / (ms / 1e3),
                "config": {"workload": f"config{cid}", "G": G, "H": H, "W": W, "K": K, "sh_degree": sh,
                           "views_per_rank": len(mine)},
                "stage_ms": {k: round(v, 4) for k, v in stage_ms.items()}, "stage_views": len(groups[0]), **extra}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# DRAM bytes of one launch, read from ncu captures of the config-2 train step (the render
# backward captured on a 4-view launch; its traffic is proportional to the views it renders).
# The Adam figure under-counts writes that were still in L2 when the kernel ended.  Re-captured
# whenever those kernels change; the capture is the one TRAFFIC_SOURCE names.
RENDER_BWD_DRAM_PER_VIEW = (179.9e6 + 36.1e6) / 4
ADAM_DRAM = 94.4e6 + 14.5e6
TRAFFIC_SOURCE = ("profiles/step_kernels_config2_4views.md (ncu, one launch per kernel, 4-view capture "
                  "at commit 99b1f18)")


def cpu_baseline_sample():
    """The oracle's whole train step on the host cores (one warm-up step that starts the workers,
    then the median of three timed steps), on the same scene as the device step."""
    from oracle.step import CpuStep, host_cores
    pkg = __graft_entry__.load_package()
    with CpuStep(pkg.synthetic.config2()) as cs:
        cs.step()
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            cs.step()
            times.append(time.perf_counter() - t0)
        step_s = float(np.median(times))
        workers, threads = cs.workers, cs.threads_per_worker
    return {"value": 1.0 / step_s, "unit": "steps/s", "cores": workers * threads, "kind": "port",
            "host_cores": host_cores(),
            "note": "numpy port of the reference path: one worker process per view, the host's cores divided over "
                    "them as BLAS threads",
            "sample": CPU_SAMPLE.format(workers=workers, threads=threads)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the timed CPU-oracle sample")
    ap.add_argument("--views", type=int, default=CONFIG["views"], help="reduced batch for profiling captures")
    ap.add_argument("--gaussians", type=int, default=CONFIG["G"], help="reduced G for profiling captures")
    ap.add_argument("--skip-e2e", action="store_true", help="skip the end-to-end and render legs (profiling)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="N > 1: gradient exchange over NVLink peer memory (default) or an NCCL all-reduce")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4],
                    help="2: the headline train step; 1 / 3 / 4: the other benchmark configs")
    args = ap.parse_args()
    if args.views != CONFIG["views"] or args.gaussians != CONFIG["G"]:
        CONFIG.update(views=args.views, G=args.gaussians,
                      workload=f"reduced profiling case: G={args.gaussians}, {args.views} views 1264x832")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    if args.config == 2:
        run_ours(args, rank, world, local_rank)
    else:
        run_config(args, rank, world, local_rank, args.config)


if __name__ == "__main__":
    main()
