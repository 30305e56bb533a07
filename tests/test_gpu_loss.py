"""Fused L1 + SSIM loss kernel vs the oracle (tools/loss_manual.py restatement + clamp)."""
import numpy as np
import pytest
import torch

from conftest import golden, rel_l2
from oracle import loss as oloss

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("case", ["l48x40", "l64x64", "l9x12"])
def test_loss_vs_reference_restatement(case, pkg):
    from tt_splat_b200 import ops
    z = golden("loss.npz")
    x, y = z[f"{case}__x"].astype(np.float32), z[f"{case}__y"].astype(np.float32)
    out = ops.loss_l1_ssim(torch.from_numpy(x).to(DEV), torch.from_numpy(y).to(DEV), 0.2, 1.0)
    assert abs(float(out["loss"][0]) - float(z[f"{case}__loss"])) < 1e-5
    assert rel_l2(out["gimg"][0].cpu().numpy(), z[f"{case}__grad"]) < 1e-3


@pytest.mark.parametrize("lam", [0.2, 0.0])
@pytest.mark.parametrize("H,W", [(64, 96), (832, 1264), (16, 16)])
def test_loss_with_clamped_inputs_vs_oracle(H, W, lam, pkg):
    """lambda 0.2 (the train step's loss) and 0 (L1 alone, a pass without SSIM work)."""
    from tt_splat_b200 import ops
    rng = np.random.default_rng(H + W)
    x = rng.uniform(-0.2, 1.2, (2, H, W, 3)).astype(np.float32)
    y = rng.uniform(0, 1, (2, H, W, 3)).astype(np.float32)
    out = ops.loss_l1_ssim(torch.from_numpy(x).to(DEV), torch.from_numpy(y).to(DEV), lam, 0.5)
    for v in range(2):
        loss, _, _, g = oloss.loss_and_grad(x[v], y[v], lam)
        assert abs(float(out["loss"][v]) - loss) < 1e-5
        assert rel_l2(out["gimg"][v].cpu().numpy(), 0.5 * g) < 1e-3


def test_loss_fn_autograd(pkg):
    from tt_splat_b200 import metrics
    rng = np.random.default_rng(1)
    x = torch.from_numpy(rng.uniform(0, 1, (40, 48, 3)).astype(np.float32)).to(DEV).requires_grad_(True)
    y = torch.from_numpy(rng.uniform(0, 1, (40, 48, 3)).astype(np.float32)).to(DEV)
    loss = metrics.loss_fn(x, y, 0.2)
    loss.backward()
    ref, _, _, g = oloss.loss_and_grad(x.detach().cpu().numpy(), y.cpu().numpy(), 0.2)
    assert abs(float(loss) - ref) < 1e-5
    assert rel_l2(x.grad.cpu().numpy(), g) < 1e-3


def test_unit_from_u8_is_correctly_rounded(pkg):
    """Every byte x expands to numpy's float32(x) / float32(255) exactly."""
    from tt_splat_b200 import ops
    bytes_ = np.tile(np.arange(256), 5)[:1023].astype(np.uint8)            # 1023: the tail path too
    out = ops.unit_from_u8(torch.from_numpy(bytes_).to(DEV)).cpu().numpy()
    assert np.array_equal(out, bytes_.astype(np.float32) / np.float32(255.0))
