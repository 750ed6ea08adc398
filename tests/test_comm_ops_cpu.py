"""Argument checks of the torch-facing comm ops (no kernel is launched on bad input)."""
import pytest
import torch

from opengda_b200.ops import comm


class _Sym:
    def __init__(self, n):
        self.local = torch.zeros(n, dtype=torch.float32)

    def ptr(self, rank=None):
        raise AssertionError("no kernel may be launched for a rejected call")


def test_out_of_range_put_and_get_are_rejected():
    s = _Sym(100)
    with pytest.raises(ValueError):
        comm.put(s, torch.zeros(101), 0)
    with pytest.raises(ValueError):
        comm.put(s, torch.zeros(10), 0, offset=4 * 95)
    with pytest.raises(ValueError):
        comm.get(torch.zeros(10), s, 0, offset=-4)
    with pytest.raises(ValueError):
        comm.put(s, torch.zeros(4, 4).t(), 0)  # not contiguous


def test_signal_op_names():
    with pytest.raises(ValueError):
        comm.signal(None, 0, 0, 1, op="xor")
