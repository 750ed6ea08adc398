"""The example-workload kernels on one GPU (the neighbour is this rank itself): the
per-phase timed loop verifies every put and stamps six phases per iteration; the fused
SAXPY + put lands a*x + y in the target and counts one arrival per CTA."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from opengda_b200.parallel import Bootstrap, Runtime
    r = Runtime(Bootstrap.create(0, 1, "127.0.0.1:0"))
    yield r
    torch.cuda.synchronize()
    r.finalize()


def test_phase_loop_verifies_and_stamps(rt):
    from opengda_b200 import native
    from opengda_b200.parallel import Barrier
    n, iters = 1 << 16, 50
    recv = rt.alloc_tensor((n,), torch.float32)
    x = torch.zeros(n, device="cuda")
    y = torch.ones(n, device="cuda")
    bar = Barrier(rt)
    stamps = torch.zeros(iters * 6, dtype=torch.int64, device="cuda")
    bad = torch.zeros(1, dtype=torch.int64, device="cuda")
    bar._b.advance(3 * iters)
    native().k_phase_loop(bar.device_ctx(), x.data_ptr(), y.data_ptr(), recv.ptr(), recv.ptr(0), n, iters, 2.0, 0, 0,
                          stamps.data_ptr(), bad.data_ptr())
    torch.cuda.synchronize()
    rt.check_device_errors()
    assert int(bad.item()) == 0
    st = stamps.view(iters, 6).cpu()
    assert bool((st[:, 1:] >= st[:, :-1]).all()) and bool((st[1:, 0] >= st[:-1, 5]).all())
    # y = 2*x + y applied once per iteration on x of that iteration: y stays finite and grew
    assert float(y[5].item()) > 1.0
    assert bar.count() == 3 * iters


def test_saxpy_put_lands_result_and_counts_ctas(rt):
    from opengda_b200 import native
    n, blocks = 1_000_003, 37
    dst = rt.alloc_tensor((n,), torch.float32)
    word = rt.signal_alloc(1)
    x = torch.rand(n, device="cuda")
    y = torch.rand(n, device="cuda")
    ref = 3.0 * x + y
    native().k_saxpy_put(x.data_ptr(), y.data_ptr(), 3.0, n, dst.ptr(0), rt.signal_peer(0, word), blocks)
    native().k_wait_count(rt.signal_local(word), blocks, rt.timeout_ns, 0)
    torch.cuda.synchronize()
    rt.check_device_errors()
    assert torch.allclose(dst.local, ref) and torch.allclose(y, ref)


def test_torch_comm_ops_put_get_signal(rt):
    from opengda_b200.ops import comm
    x = rt.alloc_tensor((1 << 16,), torch.float32)
    src = torch.arange(1 << 16, dtype=torch.float32, device="cuda")
    word = rt.signal_alloc(1)
    blocks = comm.put_signal(x, src, rt.rank, rt, word)
    comm.wait_signal(rt, word, blocks)
    assert torch.equal(x.local, src)
    back = torch.empty(1000, dtype=torch.float32, device="cuda")
    comm.get(back, x, rt.rank, offset=4 * 500)
    assert torch.equal(back, src[500:1500])
    comm.signal(rt, rt.rank, word, 5, op="add")
    comm.wait_signal(rt, word, blocks + 5, cmp="eq")
    with pytest.raises(TimeoutError):
        comm.wait_signal(rt, word, blocks + 6, timeout_ns=50_000_000)
    with pytest.raises(ValueError):
        comm.put(x, torch.zeros(1 << 17, device="cuda"), rt.rank)
    from opengda_b200 import native
    native().read_errors(True)  # the deliberate timeout above left a record
