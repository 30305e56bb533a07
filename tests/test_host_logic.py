"""Host-side logic that needs no GPU: cached binning tables, device guards, view partitions."""
import pytest
import torch


def test_cached_table_format_and_validation(pkg):
    """The reference's (idx, valid) pair -> int32 ids with -1 where invalid (valid slots first);
    holes, out-of-range ids and wrong shapes are rejected before any launch."""
    from tt_splat_b200.binned import _cached_table
    T, K, G = 3, 4, 10
    idx = torch.tensor([[5, 2, 0, 0], [9, 0, 0, 0], [0, 0, 0, 0]])
    valid = torch.tensor([[True, True, False, False], [True, False, False, False], [False] * 4])
    t = _cached_table((idx, valid), G, T, K, "cpu")
    assert t.dtype == torch.int32 and tuple(t.shape) == (1, T, K)
    assert t[0].tolist() == [[5, 2, -1, -1], [9, -1, -1, -1], [-1, -1, -1, -1]]
    hole = valid.clone()
    hole[0, 0] = False
    with pytest.raises(ValueError):
        _cached_table((idx, hole), G, T, K, "cpu")
    with pytest.raises(ValueError):
        _cached_table((idx, valid), 5, T, K, "cpu")            # id 9 >= G
    with pytest.raises(ValueError):
        _cached_table((idx[:, :3], valid[:, :3]), G, T, K, "cpu")


def test_device_guard_is_a_no_op_for_cpu_tensors(pkg):
    from tt_splat_b200._lib import on_device
    with on_device(torch.zeros(1)):
        pass
    with on_device(None):
        pass


def test_ops_reject_cpu_tensors(pkg):
    """No CPU fallback: a CPU tensor reaching an op raises before the library is called."""
    from tt_splat_b200 import ops
    with pytest.raises(RuntimeError):
        ops._dev(torch.zeros(4))
