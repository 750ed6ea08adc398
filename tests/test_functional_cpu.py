"""Argument checks of the torch.distributed-style collectives (opengda_b200.parallel.functional);
they reject bad calls before touching the GPU."""
import types

import pytest
import torch

from opengda_b200.parallel.functional import Collectives, _size_class


def _col(n=2):
    return Collectives(types.SimpleNamespace(size=n))


def test_size_classes_are_powers_of_two_multiples():
    assert _size_class(1, 8) == 8 and _size_class(9, 8) == 16 and _size_class(1024, 8) == 1024
    assert _size_class(100, 48) == 192


def test_reduction_calls_need_cuda_bf16():
    c = _col()
    with pytest.raises(TypeError):
        c.all_reduce(torch.zeros(16, dtype=torch.bfloat16))
    with pytest.raises(TypeError):
        c.reduce_scatter_tensor(torch.zeros(8), torch.zeros(16, dtype=torch.float32))


def test_all_gather_shapes_are_checked():
    c = _col(4)
    with pytest.raises(ValueError):
        c.all_gather_into_tensor(torch.zeros(15), torch.zeros(4))
    with pytest.raises(ValueError):
        c.all_gather_into_tensor(torch.zeros(12, dtype=torch.float64), torch.zeros(3))
    with pytest.raises(ValueError):  # 3 floats = 12 bytes: not a multiple of 16
        c.all_gather_into_tensor(torch.zeros(12), torch.zeros(3))
