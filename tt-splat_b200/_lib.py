"""ctypes binding of the C ABI in ``include/ttsplat_b200.h`` (``libttsplat_b200.so``).

The library is loaded on first use from this package directory (it is built in-tree by
``build.py``).  There is no fallback: a missing library, a missing CUDA device or a non-CUDA
tensor raises.  Every call passes the current torch CUDA stream, so the ops order with torch
work and can be captured in CUDA graphs.
"""
import ctypes as C
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libttsplat_b200.so")

P = C.c_void_p
I = C.c_int
F = C.c_float
D = C.c_double
SZ = C.c_size_t
U64 = C.c_uint64
LL = C.c_longlong

SIGNATURES = {
    "tts_version": (I, []),
    "tts_last_error": (C.c_char_p, []),
    "tts_read_status": (I, [P]),
    "tts_project": (I, [P, I, I, P, I, I, I, F, F, P, P, P, P, P, P, P]),
    "tts_bin_workspace_bytes": (SZ, [I, I, I, I]),
    "tts_pack_cached_workspace_bytes": (SZ, [I, I]),
    "tts_pack_cached": (I, [P, I, I, I, I, I, I, F, P, P, P, P, P, P, SZ, P]),
    "tts_bin_from_mu2d": (I, [P, P, I, I, I, I, I, I, P, P, P, P, P, SZ, P]),
    "tts_bin_from_mu2d_noalloc": (I, [P, P, I, I, I, I, I, I, P, P, P, P, P]),
    "tts_bin_pack": (I, [P, P, P, P, P, I, I, I, I, I, I, F, P, P, P, P, P, I, P, SZ, P]),
    "tts_pack_operands": (I, [P, P, P, I, I, P, P]),
    "tts_unpack_slot_grads": (I, [P, I, I, P, P, P, P]),
    "tts_render_fwd": (I, [P, I, P, I, I, I, I, P, I, P, P, P, P]),
    "tts_render_bwd": (I, [P, P, I, I, I, I, P, P, P, P, P, P, P]),
    "tts_render_fwd_rv": (I, [P, P, I, I, I, I, P, P, P, P, P]),
    "tts_render_bwd_rv": (I, [P, P, I, I, I, I, P, P, P, P, P, P, P]),
    "tts_loss_workspace_bytes": (SZ, [I, I, I]),
    "tts_loss_l1_ssim": (I, [P, P, I, I, I, F, F, P, P, P, P, SZ, P]),
    "tts_backward_workspace_bytes": (SZ, [I, I]),
    "tts_backward_params": (I, [P, I, I, P, I, I, I, I, I, F, F, F, P, P, P, P, F, F, P, P, P, P, SZ, P]),
    "tts_adam_sgld": (I, [P, P, P, P, I, I, P, P, D, D, D, F, P, U64, P]),
    "tts_step_begin": (I, [P, P]),
    "tts_adam_vec": (I, [P, P, P, P, I, P, D, D, D, D, P]),
    "tts_sgld": (I, [P, I, D, F, P, P, U64, P]),
    "tts_relocate_workspace_bytes": (SZ, [I]),
    "tts_relocate": (I, [P, P, P, I, F, F, F, P, P, P, U64, P, P, P, SZ, P]),
    "tts_sgld_relocate": (I, [P, P, P, I, P, F, P, F, F, F, P, P, P, U64, P, P, P, SZ, P]),
    "tts_peer_sgld_relocate": (I, [P, P, P, I, P, F, P, F, F, F, P, U64, P, P, P, I, I, P, SZ, P]),
    "tts_ipc_handle_bytes": (SZ, []),
    "tts_peer_alloc": (I, [SZ, C.POINTER(P)]),
    "tts_peer_free": (I, [P]),
    "tts_ipc_export": (I, [P, P]),
    "tts_ipc_open": (I, [P, C.POINTER(P)]),
    "tts_ipc_close": (I, [P]),
    "tts_peer_barrier": (I, [P, I, I, I, P, P]),
    "tts_peer_signal": (I, [P, I, I, I, P, P]),
    "tts_peer_wait": (I, [P, I, I, I, P, P]),
    "tts_adam_peer": (I, [P, P, P, P, I, I, I, I, P, P, D, D, D, P, P, P, P]),
    "tts_peer_sgld": (I, [P, I, D, F, P, P, U64, P, I, I, P]),
    "tts_spike_workspace_bytes": (SZ, [LL, LL, I]),
    "tts_quat_to_rotmat": (I, [P, LL, P, I, P]),
    "tts_quat_to_rotmat_bwd": (I, [P, P, LL, P, I, P]),
    "tts_cov3d": (I, [P, P, LL, P, I, P]),
    "tts_cov3d_bwd": (I, [P, P, P, LL, P, P, I, P]),
    "tts_project_ewa": (I, [P, P, LL, P, D, D, P, P, P, P, I, P]),
    "tts_project_ewa_bwd": (I, [P, P, LL, P, D, D, P, P, P, P, P, I, P]),
    "tts_eval_sh": (I, [I, P, I, I, P, LL, I, P, I, P]),
    "tts_eval_sh_bwd": (I, [I, P, I, I, P, LL, I, P, P, P, I, P]),
    "tts_color_from_dc": (I, [P, LL, P, P, I, P]),
    "tts_phi": (I, [P, P, LL, P, I, P]),
    "tts_phi_bwd": (I, [P, P, P, LL, P, P, I, P]),
    "tts_theta_from_conic": (I, [P, P, P, LL, LL, D, I, P, P, I, P]),
    "tts_theta_from_conic_bwd": (I, [P, P, P, LL, LL, D, P, P, P, P, I, P]),
    "tts_quad_form": (I, [P, P, P, P, LL, LL, P, I, P]),
    "tts_quad_form_bwd": (I, [P, P, P, P, P, LL, LL, P, P, P, SZ, I, P]),
    "tts_phi_theta": (I, [P, P, LL, LL, P, I, P]),
    "tts_phi_theta_bwd": (I, [P, P, P, LL, LL, P, P, P, SZ, I, P]),
    "tts_poly_splat_wgeo": (I, [P, LL, LL, D, P, P, P, I, P]),
    "tts_unit_from_u8": (I, [P, LL, P, P]),
    "tts_fma_probe_flops": (LL, [I, I]),
    "tts_fma_probe": (I, [I, I, P, P]),
    "tts_wsr_dense_fwd": (I, [P, P, P, P, P, P, P, I, I, P, P, P]),
    "tts_wsr_dense_bwd": (I, [P, P, P, P, P, P, P, I, I, P, P, P, P, P, P, P, P]),
}

_lib = None


def lib():
    """Load (once) and return the CUDA library; raises when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                               "(there is no CPU fallback)")
        h = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


class TTSError(RuntimeError):
    pass


def call(name, *args):
    """Call an entry point; raise ValueError (bad argument) or RuntimeError (CUDA/capacity)."""
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        msg = lib().tts_last_error().decode()
        if rc == 1:
            raise ValueError(f"{name}: {msg}")
        raise TTSError(f"{name}: {msg} (code {rc})")


def ptr(t):
    """Device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("tt-splat B200 ops need CUDA tensors (no CPU fallback)")
    return C.c_void_p(t.data_ptr())


def stream(device=None):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def on_device(t):
    """Context selecting a CUDA tensor's device (a no-op for anything else: the ops then raise)."""
    import contextlib
    if isinstance(t, torch.Tensor) and t.is_cuda:
        return torch.cuda.device(t.device)
    return contextlib.nullcontext()


def device_ctx(device):
    """Context selecting a torch CUDA device (a no-op for any other device)."""
    import contextlib
    device = torch.device(device)
    return torch.cuda.device(device) if device.type == "cuda" else contextlib.nullcontext()


def require_cuda():
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available: tt-splat B200 has no CPU fallback")
