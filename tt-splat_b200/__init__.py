"""tt-splat B200: matrix-native 3DGS render + train hot path on sm_100a.

The Python API mirrors the reference's ``spike`` package (``render``, ``forward``, ``backward``,
``geometry``, ``sh``, ``train``, ``mcmc``) and the binned operator pair of
``tools/m4_train_binned.py`` (``binned``); underneath, every hot op is a hand-written CUDA
kernel in ``libttsplat_b200.so`` called through its C ABI (``include/ttsplat_b200.h``).
There is no CPU fallback: the ops raise when the library or a CUDA device is missing.
"""
from . import synthetic  # noqa: F401  (numpy only)

__all__ = ["synthetic", "camera", "model", "geometry", "sh", "forward", "backward", "render",
           "binned", "train", "mcmc", "metrics", "plyio", "data", "peer", "device"]


def __getattr__(name):
    if name in __all__:
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
