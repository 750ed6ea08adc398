"""Host-side plumbing of the fused distributed GEMM, on CPU: DistGemm against a fake
runtime, with the native kernels replaced by recorders whose signatures are read from the
real bindings' docstrings -- so an argument that the binding would reject (wrong count,
a method passed where an int is due) fails here, without a GPU."""
import inspect

import pytest
import torch

import opengda_b200
from opengda_b200.models import dist_gemm


class _FakeSym:
    def __init__(self, base, n):
        self.base, self.n = base, n

    def ptr(self, rank=None):
        return self.base + (0 if rank is None else rank << 32)

    @property
    def mc_ptr(self):
        return self.base + (1 << 40)

    @property
    def local(self):
        return torch.zeros(1)


class _FakeRt:
    def __init__(self, n=2, rank=0, mc=True):
        self.size, self.rank, self.multicast_supported = n, rank, mc
        self.timeout_ns = 10 ** 9
        self._next = 1 << 20

    def alloc_tensor(self, shape, dtype=torch.bfloat16, multicast=False, exchange=True):
        self._next += 1 << 30
        return _FakeSym(self._next, self.size)

    def exchange(self):
        pass

    def signal_alloc(self, n):
        return 64

    def signal_peer(self, rank, word=0):
        return (rank + 1) << 36 | word * 8

    def signal_local(self, word=0):
        return self.signal_peer(self.rank, word)

    def signal_multicast(self, word=0):
        return 1 << 44 | word * 8


def _params(doc: str):
    head = doc.strip().splitlines()[0]
    inner = head[head.index("(") + 1:head.rindex(")")]
    parts, depth, cur = [], 0, ""
    for ch in inner:  # split on the commas outside brackets
        depth += ch == "["
        depth -= ch == "]"
        if ch == "," and depth == 0:
            parts.append(cur)
            cur = ""
        else:
            cur += ch
    parts.append(cur)
    return [(p.split(":")[0].strip(), "=" in p) for p in parts if p.strip()]


class _Recorder:
    def __init__(self, real):
        self.calls = []
        self.sig = {}
        for name in ("k_ag_gemm", "k_gemm_rs"):
            params = _params(getattr(real, name).__doc__)
            self.sig[name] = inspect.Signature([
                inspect.Parameter(p, inspect.Parameter.POSITIONAL_OR_KEYWORD, default=0 if d else inspect._empty)
                for p, d in params])

    def __getattr__(self, name):
        sig = self.sig[name]

        def call(*args, **kw):
            bound = sig.bind(*args, **kw)
            for k, v in bound.arguments.items():
                assert isinstance(v, (int, list)), (name, k, type(v))
                if isinstance(v, list):
                    assert all(isinstance(x, int) for x in v), (name, k)
            self.calls.append((name, dict(bound.arguments)))
        return call


@pytest.mark.parametrize("mode,nvls", [("ag", True), ("ag", False), ("rs", True), ("rs", False)])
def test_fused_dist_gemm_passes_binding_compatible_arguments(monkeypatch, mode, nvls):
    real = opengda_b200.native()
    rec = _Recorder(real)
    monkeypatch.setattr(opengda_b200, "native", lambda: rec)
    M = N = K = 1024
    rt = _FakeRt(2, 0, mc=True)
    m = dist_gemm.DistGemm(M, N, K, mode, rt=rt, device=torch.device("cpu"), nvls=nvls)
    A = torch.zeros(*m.a_shape(), dtype=torch.bfloat16)
    B = torch.zeros(*m.b_shape(), dtype=torch.bfloat16)
    if mode == "ag":
        m.a_slot = lambda parity=None: A  # zero-copy slot: no copy on the fake buffers
    for _ in range(3):
        m(A, B)
    assert [c[0] for c in rec.calls] == ["k_" + ("ag_gemm" if mode == "ag" else "gemm_rs")] * 3
    args = rec.calls[-1][1]
    assert args["epoch"] == 3
    if mode == "ag":
        assert (args["a_mc"] != 0) == bool(nvls) and (args["arrivals_mc"] != 0) == bool(nvls)
        assert args["tile_counter"] != 0 and args["comm_ctas"] > 0
    else:
        assert (args.get("staging_mc", 0) != 0) == bool(nvls)
        if nvls:
            assert args["band_tiles"] != 0 and args["tile_counter"] != 0


def test_counter_settings_are_frozen_after_the_first_call(monkeypatch):
    real = opengda_b200.native()
    rec = _Recorder(real)
    monkeypatch.setattr(opengda_b200, "native", lambda: rec)
    m = dist_gemm.DistGemm(1024, 1024, 1024, "ag", rt=_FakeRt(2, 0), device=torch.device("cpu"), nvls=True)
    A = torch.zeros(*m.a_shape(), dtype=torch.bfloat16)
    B = torch.zeros(*m.b_shape(), dtype=torch.bfloat16)
    m.a_slot = lambda parity=None: A
    m(A, B)
    m.comm_ctas = 24  # free to change
    m(A, B)
    m.units_per_band = 8
    with pytest.raises(ValueError, match="units_per_band"):
        m(A, B)


@pytest.mark.parametrize("mode,n,nvls,want", [("ag", 2, True, 2), ("ag", 4, True, 2), ("ag", 8, True, 1),
                                              ("rs", 8, True, 2), ("rs", 2, False, 0), ("ag", 2, False, 2)])
def test_tile_choice_by_shape(monkeypatch, mode, n, nvls, want):
    """256 x 512 CTA-pair tiles where they fill the 74 CTA pairs about as evenly as 128 x 256
    tiles fill the 148 SMs (16384^3: yes at 2 and 4 GPUs; not for the all-gather at 8, whose
    2048-column shard gives 256 such tiles = 3.5 waves, so 256 x 256 pair tiles there); the
    unicast reduce-scatter has no pair variant.  GICC_DIST_GEMM_PAIR overrides the choice."""
    monkeypatch.delenv("GICC_DIST_GEMM_PAIR", raising=False)
    m = dist_gemm.DistGemm(16384, 16384, 16384, mode, rt=_FakeRt(n, 0, mc=True), device=torch.device("cpu"),
                           nvls=nvls)
    assert m.pair == want
    monkeypatch.setenv("GICC_DIST_GEMM_PAIR", "1")
    m = dist_gemm.DistGemm(16384, 16384, 16384, mode, rt=_FakeRt(n, 0, mc=True), device=torch.device("cpu"),
                           nvls=nvls)
    assert m.pair == (1 if (mode == "ag" or nvls) else 0)
