"""Peer-memory exchange between the ranks of one node (the multi-GPU optimizer step).

Each rank allocates one region in its GPU with ``tts_peer_alloc`` holding its parameter
vector, gradient vector, loss and barrier flags; the regions are exported as CUDA IPC handles,
exchanged over the process group (a host all-gather of bytes) and opened by every other rank,
so each rank holds device pointers to all N regions.  ``tts_adam_peer`` then reduces and
updates one shard per rank and writes the result into every region over NVLink, between two
``tts_peer_barrier`` kernels.  The regions are used as torch tensors through the CUDA array
interface (no copy).
"""
import ctypes as C

import torch

from ._lib import call, lib

_ALIGN = 256
FLAG_INTS = 32             # 2 phases x 8 ranks, the Adam block counter, padding


def _round(n):
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


class _Cai:
    """Minimal __cuda_array_interface__ holder for a raw device pointer."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None, "stream": None}


def _view(ptr, n, dtype, device):
    typestr = {torch.float32: "<f4", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_Cai(ptr, (n,), typestr), device=device)


def layout(n_params):
    """Byte offsets of the parameter vector, gradient vector, loss and flags in a region."""
    off_p = 0
    off_g = off_p + _round(4 * n_params)
    off_l = off_g + _round(4 * n_params)
    off_f = off_l + _ALIGN
    return off_p, off_g, off_l, off_f, off_f + _round(4 * FLAG_INTS)


def shard_range(n, rank, world):
    """Elements [lo, hi) of a length-n vector owned by ``rank`` (the split of tts_adam_peer:
    equal chunks rounded up to whole 16-byte vectors, the last chunk shorter)."""
    chunk = (-(-n // world) + 3) // 4 * 4
    lo = min(n, rank * chunk)
    return lo, min(n, lo + chunk)


class PeerRegions:
    """This rank's region plus the opened regions of its peers (index = rank)."""

    def __init__(self, n_params, device, group):
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the peer optimizer step supports up to 8 ranks (one node)")
        self.n = int(n_params)
        self.off = layout(self.n)
        ptr = C.c_void_p()
        call("tts_peer_alloc", self.off[4], C.byref(ptr))
        self.base = ptr.value
        hb = lib().tts_ipc_handle_bytes()
        h = (C.c_char * hb)()
        call("tts_ipc_export", C.c_void_p(self.base), h)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h), group=group)
        self.bases = []
        for r, hr in enumerate(handles):
            if r == self.rank:
                self.bases.append(self.base)
                continue
            buf = (C.c_char * hb).from_buffer_copy(hr)
            p = C.c_void_p()
            call("tts_ipc_open", buf, C.byref(p))
            self.bases.append(p.value)
        self.params = _view(self.base + self.off[0], self.n, torch.float32, device)
        self.grads = _view(self.base + self.off[1], self.n, torch.float32, device)
        self.loss = _view(self.base + self.off[2], 1, torch.float32, device)

        def table(k, ctype):
            return (ctype * self.world)(*[ctype(b + self.off[k]) for b in self.bases])
        self.t_params = table(0, C.c_void_p)
        self.t_grads = table(1, C.c_void_p)
        self.t_loss = table(2, C.c_void_p)
        self.t_flags = table(3, C.c_void_p)

    def close(self):
        """Unmap the peers' regions and free this one (every rank calls it; a barrier first
        makes sure no peer still writes into this rank's region)."""
        import torch.distributed as dist
        if self.base is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for r, b in enumerate(self.bases):
            if r != self.rank:
                call("tts_ipc_close", C.c_void_p(b))
        dist.barrier(group=self.group)
        call("tts_peer_free", C.c_void_p(self.base))
        self.base = None
