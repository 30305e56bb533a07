"""Run-device selection (mirrors spike/device.py:13-23 for a CUDA-only library).

The reference resolves CUDA when available and falls back to the CPU.  Every op of this package
runs on the GPU and none has a CPU path, so ``default_device`` resolves a CUDA device or raises:
an explicit ``"cpu"`` is refused with ``ValueError``, and CUDA requested (or needed) without a
visible device raises ``RuntimeError`` right away instead of at the first launch.
"""
import torch


def default_device(override=None):
    """``override`` ("cuda", "cuda:1", a torch.device) wins; otherwise the current CUDA device."""
    dev = torch.device(override) if override else torch.device("cuda")
    if dev.type != "cuda":
        raise ValueError(f"device '{dev}': tt-splat B200 runs on CUDA devices only (no CPU path)")
    if not torch.cuda.is_available():
        raise RuntimeError(f"device '{dev}' requested but CUDA is unavailable")
    return dev
