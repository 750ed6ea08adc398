"""The CUDA-graph capture guard (opengda_b200.utils.graphs), with the capture state faked."""
import pytest

from opengda_b200.utils import graphs


def test_refuse_capture_only_while_capturing(monkeypatch):
    monkeypatch.setattr(graphs, "capturing", lambda: False)
    graphs.refuse_capture("X")  # not capturing: no error
    monkeypatch.setattr(graphs, "capturing", lambda: True)
    with pytest.raises(RuntimeError, match="X cannot be captured"):
        graphs.refuse_capture("X")


def test_capturing_is_false_without_a_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    assert graphs.capturing() is False
