"""The topology probe's logic against a fake NVML and fake P2P tables (no GPU)."""
from opengda_b200.utils.topology import probe


class FakeNvml:
    def __init__(self, links_per_gpu):
        self.links = links_per_gpu
        self.calls = []

    def nvmlInit(self):
        self.calls.append("init")

    def nvmlShutdown(self):
        self.calls.append("shutdown")

    def nvmlDeviceGetCount(self):
        return len(self.links)

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetName(self, h):
        return b"NVIDIA B200"

    def nvmlDeviceGetNvLinkState(self, h, link):
        if link >= 18:
            raise RuntimeError("no such link")
        return 1 if link < self.links[h] else 0

    def nvmlDeviceGetNvLinkVersion(self, h, link):
        return 5


def _pairs(n, access=1, atomics=1, rank=lambda s, d: 0):
    return lambda: [{"src": s, "dst": d, "access": access, "native_atomics": atomics, "array_access": 1,
                     "perf_rank": rank(s, d)} for s in range(n) for d in range(n) if s != d]


def test_uniform_nvswitch_node():
    nv = FakeNvml([18] * 8)
    res = probe(nvml=nv, p2p=_pairs(8))
    assert res["uniform"] and not res["pairs_without_access"]
    assert len(res["p2p"]) == 56
    assert [g["active_links"] for g in res["nvlink"]] == [18] * 8 and res["nvlink"][0]["versions"] == [5]
    assert nv.calls == ["init", "shutdown"]  # read-only queries, NVML released


def test_non_uniform_and_missing_access_are_reported():
    res = probe(nvml=None, p2p=_pairs(4, rank=lambda s, d: abs(s - d)))
    assert not res["uniform"] and res["nvlink"] is None
    res = probe(nvml=None, p2p=_pairs(2, access=0))
    assert not res["uniform"] and res["pairs_without_access"] == [(0, 1), (1, 0)]


def test_unusable_nvml_is_reported_not_raised():
    class Broken(FakeNvml):
        def nvmlInit(self):
            raise RuntimeError("no permission")
    res = probe(nvml=Broken([18]), p2p=_pairs(2))
    assert res["nvlink"] is None and "no permission" in res["nvml_error"] and res["uniform"]


def test_single_gpu_is_not_called_uniform():
    assert probe(nvml=None, p2p=_pairs(1))["uniform"] is False


import pytest  # noqa: E402


@pytest.mark.gpu
def test_probe_on_this_node():
    import torch
    n = torch.cuda.device_count()
    res = probe()
    assert len(res["p2p"]) == n * (n - 1)
    if n > 1:
        assert res["uniform"], res  # an NVSwitch node: every pair equal
    if res["nvlink"] is not None:
        assert len(res["nvlink"]) >= n


def test_environment_summary_runs_without_gpu():
    from opengda_b200.utils.topology import environment
    env = environment()
    assert env["python"] and env["native_library"] == "loaded"
