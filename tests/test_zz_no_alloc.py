"""The allocation-free binning entry point against the allocating one.

Callers that cannot allocate device memory while they bin (inside CUDA-graph stream capture, or
inside a host runtime that owns the device allocator) use ``tts_bin_from_mu2d_noalloc``, whose
scratch lives in a static device array.  Its tables must equal those of ``tts_bin_from_mu2d``
bit for bit (the tolerance every binning test uses), also on a second call that reuses the
static scratch left over from the first.  This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(pkg, seed, G, H, W):
    mu, keep = pkg.synthetic.stress_mu2d(seed, G, H, W, n_clusters=12, sigma_px=9.0, n_special=8)
    return (torch.from_numpy(mu).to(DEV).contiguous(),
            torch.from_numpy(keep.astype(np.uint8)).to(DEV).contiguous())


def _outputs(G, T, K, S):
    return (torch.full((1, T, K), 7, dtype=torch.int32, device=DEV),
            torch.full((1, T), 7, dtype=torch.int32, device=DEV),
            torch.full((1, T), 7, dtype=torch.int32, device=DEV),
            torch.full((1, G, S), 7, dtype=torch.int32, device=DEV))


def test_noalloc_binning_equals_allocating_entry_point_twice(pkg):
    from tt_splat_b200 import _lib
    lib = _lib.lib()
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    H, W, R, K = 256, 320, 1, 64
    T, S = (H // 16) * (W // 16), (2 * R + 1) ** 2
    for seed, G in ((301, 30000), (302, 12000)):
        mu, keep = _inputs(pkg, seed, G, H, W)
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        ref = _outputs(G, T, K, S)
        nbytes = lib.tts_bin_workspace_bytes(G, 1, H, W)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
        rc = lib.tts_bin_from_mu2d(p(mu), p(keep), G, 1, H, W, R, K, *(p(t) for t in ref), p(ws), nbytes, stream)
        assert rc == 0, lib.tts_last_error()
        got = _outputs(G, T, K, S)
        rc = lib.tts_bin_from_mu2d_noalloc(p(mu), p(keep), G, 1, H, W, R, K, *(p(t) for t in got), stream)
        assert rc == 0, lib.tts_last_error()
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
        assert int(ref[2].sum()) > 0 and int((ref[2] > K).sum()) > 0     # overflowing tiles exercised


def test_noalloc_rejects_problems_beyond_its_static_scratch(pkg):
    from tt_splat_b200 import _lib
    lib = _lib.lib()
    G = 2_000_000                                     # ~48 MB of scratch > the 16 MiB array
    rc = lib.tts_bin_from_mu2d_noalloc(None, None, G, 1, 1072, 1920, 1, 256, None, None, None, None, None)
    assert rc == 3 and b"static buffer" in lib.tts_last_error()
