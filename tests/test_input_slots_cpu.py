"""DistGemm.input_slots(): the A slots of the next two calls, in call order, for the fused
all-gather mode (what HostFeeder fills zero-copy); None where the mode does not
double-buffer its input.  Checked on the host with stand-in slot buffers."""
import types

import torch

from opengda_b200.models.dist_gemm import DistGemm


def _model(epoch, fused=True, mode="ag", world=2, rank=1):
    m = DistGemm.__new__(DistGemm)
    m.fused, m.mode, m.world, m.rank, m.epoch = fused, mode, world, rank, epoch
    m.M, m.K = 8, 4
    m.A_bufs = [types.SimpleNamespace(local=torch.full((m.M, m.K), float(p))) for p in range(2)]
    m.A_full = types.SimpleNamespace(local=torch.full((m.M, m.K), 9.0))
    return m


def test_slots_follow_the_call_parity():
    for epoch in range(5):
        m = _model(epoch)
        s = m.input_slots()
        # call e uses parity e % 2 (forward increments epoch before choosing the slot)
        assert [int(t[0, 0]) for t in s] == [(epoch + 1) % 2, (epoch + 2) % 2]
        assert all(t.shape == (m.M // m.world, m.K) for t in s)
        assert s[0].data_ptr() == m.a_slot().data_ptr()  # a_slot() is the next call's slot


def test_no_slots_where_input_is_not_double_buffered():
    assert _model(0, fused=False).input_slots() is None
    assert _model(0, mode="rs").input_slots() is None
    assert _model(0, world=1).input_slots() is None
