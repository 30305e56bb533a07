"""The N > 1 host logic on CPU: two gloo ranks split the view batch with partition_views, compute
their (oracle) gradients with the 1/n_views scale, and reduce_across_ranks makes every rank hold
the single-process gradient and loss.  No GPU; the same functions run under NCCL in TrainStep."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scene():
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    return pkg, pkg.synthetic.config2(seed=7, G=400, H=32, W=48, n_views=3)


def _rank_grads(views, n_total):
    from oracle import loss as oloss, pipeline
    pkg, sc = _scene()
    p = sc["params"]
    flat = np.zeros(59 * 400 + 1)
    loss_sum = 0.0
    for v in views:
        fw = pipeline.render_view(p, 3, sc["cams"][v], K=32)
        lv, _, _, g = oloss.loss_and_grad(fw["img"], sc["targets"][v], 0.2)
        loss_sum += lv
        gv = pipeline.backward_view(fw, (g / n_total).astype(np.float32), p, 3)
        parts = [gv[n].reshape(-1) for n in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc", "color_rest")]
        flat += np.concatenate(parts + [np.array([gv["w_b_raw"]])])
    return flat, loss_sum


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import __graft_entry__
        pkg = __graft_entry__.load_package()
        from tt_splat_b200.train import partition_views, reduce_across_ranks
        views = partition_views(3, world, rank)
        g, l = _rank_grads(views, 3)
        gt = torch.from_numpy(g)
        lt = torch.tensor([l], dtype=torch.float64)
        reduce_across_ranks(gt, lt)
        out[rank] = (gt.numpy().copy(), float(lt[0]))
    finally:
        dist.destroy_process_group()


def test_partition_views():
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from tt_splat_b200.train import partition_views
    assert partition_views(8, 1, 0) == list(range(8))
    assert [partition_views(8, 4, r) for r in range(4)] == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert [partition_views(3, 2, r) for r in range(2)] == [[0, 1], [2]]
    assert sum(len(partition_views(5, 8, r)) for r in range(8)) == 5


def test_two_gloo_ranks_reduce_to_the_single_process_gradient():
    world = 2
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
    full_g, full_l = _rank_grads([0, 1, 2], 3)
    for r in range(world):
        g, l = out[r]
        assert np.abs(g - full_g).max() <= 1e-9 * max(1.0, np.abs(full_g).max())
        assert abs(l - full_l) < 1e-9
    assert np.array_equal(out[0][0], out[1][0])      # replicas see the same bits


def _replica_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import __graft_entry__
        __graft_entry__.load_package()
        from tt_splat_b200.train import replicas_agree
        flat = torch.from_numpy(np.random.default_rng(3).standard_normal(59 * 300 + 1).astype(np.float32))
        same = replicas_agree(flat)
        if rank == 1:                                    # a planted one-ulp divergence on one rank
            flat[1234] = float(np.nextafter(flat[1234].numpy(), np.float32(np.inf)))
        out[rank] = (same, replicas_agree(flat))
    finally:
        dist.destroy_process_group()


def test_replica_check_detects_a_one_ulp_divergence():
    world = 2
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_replica_worker, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
    assert [out[r] for r in range(world)] == [(True, False), (True, False)]
