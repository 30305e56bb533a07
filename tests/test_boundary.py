"""The C-ABI boundary on the CPU: the library loads, exports every declared symbol, the ctypes
binding matches the header, and host-side validation raises the reference's error kinds
without touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import REPO

HDR = os.path.join(REPO, "include", "ttsplat_b200.h")


def declared():
    txt = open(HDR).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|long long|const char\*)\s+(tts_\w+)\(", txt, re.M)))


def test_library_exports_every_declared_symbol(pkg):
    from tt_splat_b200 import _lib
    lib = _lib.lib()
    names = declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (tts_\w+)", out))
    assert set(names) <= exported


def test_binding_matches_header(pkg):
    from tt_splat_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared()
    txt = open(HDR).read().replace("\n", " ")
    for name, (_, args) in _lib.SIGNATURES.items():
        m = re.search(rf"(?:int|size_t|long long|char\*|void)\s+\**{name}\(([^)]*)\);", txt)
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), name


def test_host_queries_and_validation(pkg):
    from tt_splat_b200 import _lib
    lib = _lib.lib()
    assert lib.tts_version() == 1
    assert lib.tts_bin_workspace_bytes(1000, 2, 64, 64) > 0
    assert lib.tts_loss_workspace_bytes(1, 64, 64) > 0
    assert lib.tts_relocate_workspace_bytes(1000) > 0
    # invalid sizes are rejected before any launch (null device pointers are never touched)
    rc = lib.tts_render_fwd(None, 0, None, 1, 15, 16, 128, None, 1, None, None, None, None)
    assert rc == 1 and b"multiples of 16" in lib.tts_last_error()
    rc = lib.tts_bin_from_mu2d(None, None, 10, 1, 16, 16, 1, 300, None, None, None, None, None, 0, None)
    assert rc == 1 and b"K" in lib.tts_last_error()
    rc = lib.tts_bin_from_mu2d(None, None, 10, 1, 16, 16, 1, 8, None, None, None, None, None, 0, None)
    assert rc == 3   # workspace too small


def test_cpu_tensors_are_refused(pkg):
    import torch
    from tt_splat_b200 import ops
    flat = torch.zeros(59 * 4 + 1)
    cams = torch.zeros(1, 20)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.project(flat, 4, 0, cams, 16, 16)
    with pytest.raises(RuntimeError):
        ops.loss_l1_ssim(torch.zeros(16, 16, 3), torch.zeros(16, 16, 3))


def test_reference_error_kinds(pkg):
    from tt_splat_b200 import binned, ops, render
    with pytest.raises(ValueError, match="unknown arm"):
        render.render(None, None, arm="Z")
    with pytest.raises(AssertionError):
        binned.TileMap(100, 64, device="cpu")
    with pytest.raises(AssertionError):
        ops.tiles(1080, 1920)


def test_product_never_imports_oracle():
    pkgdir = os.path.join(REPO, "tt-splat_b200")
    for root, _, files in os.walk(pkgdir):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh")):
                txt = open(os.path.join(root, f)).read()
                assert "import oracle" not in txt and "from oracle" not in txt, f
