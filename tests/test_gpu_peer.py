"""The NVLink peer-memory optimizer step.

* A barrier whose peer never signals gives up after its bounded wait and reports it in the
  status word (the failure is a flag nothing sets; no fault, the context stays usable).
* On two GPUs, training steps with the peer exchange (shard reduce + Adam + peer broadcast)
  equal bit for bit the same steps with an NCCL all-reduce and replicated Adam: with two ranks
  both sum the two gradients in one addition, and the Adam arithmetic is the same.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_barrier_times_out_and_reports_status(pkg):
    from tt_splat_b200 import _lib
    lib = _lib.lib()
    st = ctypes.c_int(0)
    lib.tts_read_status(ctypes.byref(st))                     # clear
    flags = torch.zeros(2, 16, dtype=torch.int32, device=DEV)
    table = (ctypes.c_void_p * 2)(flags[0].data_ptr(), flags[1].data_ptr())
    epoch = torch.ones(1, dtype=torch.int32, device=DEV)
    # rank 0 of 2: "rank 1" is a local buffer nobody writes, so the wait runs out
    rc = lib.tts_peer_barrier(table, 0, 2, 0, ctypes.c_void_p(epoch.data_ptr()),
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    lib.tts_read_status(ctypes.byref(st))
    assert st.value & 4
    assert int(flags[0, 0]) == 1 and int(flags[1, 0]) == 1  # the signals went out
    x = torch.ones(4, device=DEV) * 2                        # the context is still usable
    assert float(x.sum()) == 8.0


def test_train_step_raises_after_a_timed_out_wait(pkg):
    """A peer wait that ran out sets the status word; the train step's status check (called by
    check_replicas and at the end of fit / train_mcmc) raises naming it, then the word is clear."""
    from tt_splat_b200 import camera, model, ops, train
    ops.read_status()                                         # clear
    sc = pkg.synthetic.config2(seed=5, G=500, H=32, W=48, n_views=1)
    m = model.GaussianModel.from_arrays(sc["params"], device=DEV)
    st = train.TrainStep(m, [camera.Camera.from_dict(sc["cams"][0])], sc["targets"], sh_degree=3, use_graph=False)
    st.step()
    st.check_status()                                         # a clean step: no error
    flags = torch.zeros(2, 16, dtype=torch.int32, device=DEV)
    table = (ctypes.c_void_p * 2)(flags[0].data_ptr(), flags[1].data_ptr())
    epoch = torch.ones(1, dtype=torch.int32, device=DEV)
    assert ops.lib().tts_peer_wait(table, 0, 2, 0, ctypes.c_void_p(epoch.data_ptr()),
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    with pytest.raises(RuntimeError, match="peer-exchange wait timed out"):
        st.check_replicas()
    st.check_status()                                         # read and cleared


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        import __graft_entry__
        pkg = __graft_entry__.load_package()
        from tt_splat_b200 import camera, model, train
        sc = pkg.synthetic.config2(seed=11, G=6000, H=96, W=128, n_views=4)
        mine = train.partition_views(4, world, rank)
        res = {}
        for exchange in ("peer", "nccl"):
            m = model.GaussianModel.from_arrays(sc["params"], device="cuda")
            cams = [camera.Camera.from_dict(sc["cams"][i]) for i in mine]
            st = train.TrainStep(m, cams, [sc["targets"][i] for i in mine], sh_degree=3, noise_lr=5e5,
                                 relocate_every=2, dead_frac=0.01, offset=0.005, lambda_o=0.01, lambda_s=0.01,
                                 seed=3, n_views_total=4, process_group=dist.group.WORLD, exchange=exchange)
            losses = [float(st.step()) for _ in range(5)]
            torch.cuda.synchronize()
            agree = train.replicas_agree(st.flat, dist.group.WORLD)
            res[exchange] = (st.flat.detach().cpu().numpy().copy(), losses, agree)
            st.release()
        out[rank] = res
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_equals_nccl_allreduce_on_two_gpus():
    import torch.multiprocessing as mp
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    for r in range(world):
        (pp, lp, ap), (pn, ln, an) = out[r]["peer"], out[r]["nccl"]
        assert ap and an
        assert lp == ln
        assert np.array_equal(pp, pn)
    assert np.array_equal(out[0]["peer"][0], out[1]["peer"][0])
