import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
for _p in (REPO, GOLDEN):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import __graft_entry__  # noqa: E402

ttsplat = __graft_entry__.load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def golden(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


def cam_from(z, prefix="cam_"):
    intr = z[prefix + "intr"]
    hw = z[prefix + "hw"]
    return dict(R_v=z[prefix + "R_v"].astype(np.float32), t_v=z[prefix + "t_v"].astype(np.float32),
                fx=float(intr[0]), fy=float(intr[1]), cx=float(intr[2]), cy=float(intr[3]),
                H=int(hw[0]), W=int(hw[1]))


def params_from(z, G=None):
    p = {k: z[k].astype(np.float32) for k in ("means3d", "log_scales", "quats", "opacity_raw", "color_dc")}
    Gn = p["means3d"].shape[0]
    p["color_rest"] = z["color_rest"].astype(np.float32) if "color_rest" in z else np.zeros((Gn, 15, 3), np.float32)
    p["w_b_raw"] = np.float32(z["w_b_raw"])
    return p


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="session")
def pkg():
    return ttsplat
