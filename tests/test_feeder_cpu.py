"""HostFeeder's consumer-buffer mode (zero-copy input into DistGemm.input_slots()): buffers of
the wrong shape, dtype or number are rejected before any stream or event is made."""
import pytest
import torch

from opengda_b200.utils.feeder import HostFeeder


@pytest.mark.parametrize("bufs", [
    [torch.empty(4, 8)],                                  # one buffer: nothing to double-buffer
    [torch.empty(4, 8), torch.empty(4, 9)],               # shape
    [torch.empty(4, 8), torch.empty(4, 8, dtype=torch.float16)],  # dtype
])
def test_feeder_rejects_unsuitable_buffers(bufs):
    with pytest.raises(ValueError):
        HostFeeder((4, 8), torch.float32, torch.device("cpu"), bufs=bufs)
