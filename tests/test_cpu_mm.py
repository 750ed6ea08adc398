"""Distributed matmul on CPU gloo ranks (fp32 1024^3): row-block A, broadcast B, gathered C, rtol 1e-5."""
from opengda_b200.models.cpu_mm import run


def test_cpu_distributed_matmul_world2():
    res = run(2)
    assert res.get("ok") is True, res
