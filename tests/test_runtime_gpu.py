"""Single-GPU tests of the runtime: symmetric allocation, host-queued puts + device flush,
barrier kernels, pattern checks and a bounded wait that must time out cleanly."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from opengda_b200.parallel import Bootstrap, Runtime
    boot = Bootstrap.create(0, 1, "127.0.0.1:0")
    r = Runtime(boot)
    yield r
    torch.cuda.synchronize()
    r.finalize()


def _n():
    from opengda_b200 import native
    return native()


def test_symmetric_tensor_and_remote_ptr(rt):
    t = rt.alloc_tensor((1024, 64), torch.float32)
    t.local.copy_(torch.arange(1024 * 64, dtype=torch.float32, device="cuda").view(1024, 64))
    assert t.peer(0).data_ptr() == t.local.data_ptr()
    addr, rkey = rt.remote_buffer(0, t.index)
    assert addr == t.ptr() and rkey == t.index
    assert t.local.sum().item() == float(sum(range(1024 * 64)))


def test_register_cudamalloc_tensor(rt):
    x = torch.randn(4096, device="cuda")
    b = rt.register_buffer(x)
    rt.exchange()
    assert b["ptr"] == x.data_ptr() and b["index"] == rt.native.num_buffers - 1
    assert rt.native.remote_ptr(0, b["index"], 16) == x.data_ptr() + 16


def test_put_no_db_flush_wait(rt):
    src = rt.alloc_tensor((1 << 20,), torch.uint8)
    dst = rt.alloc_tensor((1 << 20,), torch.uint8)
    n = _n()
    n.k_fill_pattern(src.ptr(), 1 << 20, 17)
    dst.local.zero_()
    torch.cuda.synchronize()
    rt.reset()
    toks = [rt.put_no_db(src.index, 0, dst.index, 1 << 18, src_off=i << 18, dst_off=i << 18) for i in range(4)]
    ctx = rt.prepare_trigger(toks[-1])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    n.k_flush(ctx, status.data_ptr())
    for t in toks:
        rt.wait(t)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert torch.equal(src.local, dst.local)


def test_barrier_single_and_continuous(rt):
    from opengda_b200.parallel import Barrier
    b = Barrier(rt)
    flag = torch.zeros(1, dtype=torch.int64, device="cuda")
    b.run_single(flag.data_ptr())
    b.wait_completion()
    assert flag.item() == 42 and b.count() == 1
    cnt = torch.zeros(1, dtype=torch.int64, device="cuda")
    b.run_continuous(1000, cnt.data_ptr())
    b.wait_continuous()
    torch.cuda.synchronize()
    assert cnt.item() == 1000 and b.count() == 1001
    rt.check_device_errors()


def test_copy_pattern_roundtrip():
    n = _n()
    for nbytes in (1, 15, 16, 1000, 1 << 20, (1 << 24) + 3):
        a = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        b = torch.zeros(nbytes + 1, dtype=torch.uint8, device="cuda")
        n.k_fill_pattern(a.data_ptr(), nbytes, nbytes)
        n.k_copy(b.data_ptr() + 1, a.data_ptr(), nbytes)  # misaligned destination path
        bad = torch.zeros(1, dtype=torch.int64, device="cuda")
        n.k_check_pattern(b.data_ptr() + 1, nbytes, nbytes, bad.data_ptr())
        torch.cuda.synchronize()
        assert bad.item() == 0, nbytes


def test_bounded_wait_times_out_and_context_survives():
    """A wait on a flag that nobody sets ends with ETIMEDOUT; the GPU context stays usable."""
    n = _n()
    n.read_errors(True)
    flag = torch.zeros(1, dtype=torch.int64, device="cuda")
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    n.k_wait_signal(flag.data_ptr(), 2, 1, 50_000_000, status.data_ptr())  # CMP_GE 1, 50 ms
    torch.cuda.synchronize()
    assert status.item() == 1  # GICC_ETIMEDOUT
    rec = n.read_errors(True)
    assert rec["status"] == "ETIMEDOUT" and rec["where"] == "signal_wait" and rec["expected"] == 1
    # context still healthy
    x = torch.randn(1000, device="cuda")
    assert torch.isfinite(x.sum()).item()
    n.k_signal(flag.data_ptr(), 5, 0)
    n.k_wait_signal(flag.data_ptr(), 2, 5, 50_000_000, status.data_ptr())
    torch.cuda.synchronize()
    assert status.item() == 0


def test_nvshmem_style_api(rt):
    from opengda_b200.parallel import api
    api.init(rt)
    p = api.malloc(1 << 16)
    assert api.remote_ptr(p, 0) == p and api.my_pe() == 0 and api.n_pes() == 1
    assert api.context() != 0
    api.barrier()


def test_active_messages_to_self(rt):
    from opengda_b200.parallel.am import Am, CHECKSUM, COUNTER_ADD, ECHO
    am = Am(rt, nslots=4, max_payload=512)
    for i in range(10):  # more messages than slots: the poll returns credit
        assert am.send_handle(0, COUNTER_ADD, [i + 1]) > 0
        assert am.poll_once() == 1
    assert am.counter() == sum(range(1, 11))
    am.send_payload(0, CHECKSUM, [0], bytes(range(200)))
    assert am.poll_once() == 1 and am.checksum() == sum(range(200))
    seq = am.send_handle(0, ECHO, [1234], request=True)
    assert am.poll_once() == 1
    assert am.wait_reply(0, seq) == 1234


def test_bounds_checked_put_records_erange_and_skips(rt, monkeypatch):
    """GICC_CHECKS=1: an out-of-range put through a DeviceCtx is refused and recorded."""
    n = _n()
    src = rt.alloc_tensor((4096,), torch.uint8)
    dst = rt.alloc_tensor((4096,), torch.uint8)
    src.local.fill_(7)
    dst.local.zero_()
    monkeypatch.setenv("GICC_CHECKS", "1")
    ctx = rt.prepare(0, dst.index)
    n.read_errors(True)
    # in range: lands
    n.k_ctx_put(ctx, src.ptr(), src.index, dst.ptr(0), dst.index, 1024)
    torch.cuda.synchronize()
    assert n.read_errors(True)["code"] == 0 and int(dst.local[:1024].sum()) == 7 * 1024
    # past the end of the destination: refused, nothing written beyond
    dst.local.zero_()
    n.k_ctx_put(ctx, src.ptr(), src.index, dst.ptr(0) + 4000, dst.index, 1024)
    torch.cuda.synchronize()
    rec = n.read_errors(True)
    assert rec["status"] == "ERANGE" and rec["where"] == "bounds"
    assert int(dst.local.sum()) == 0


def test_host_put_get(rt):
    a = rt.alloc_tensor((1 << 20,), torch.uint8)
    x = torch.randint(0, 255, (1 << 20,), dtype=torch.uint8, device="cuda")
    rt.native.host_put(x.data_ptr(), 0, a.index, 0, 1 << 20)
    y = torch.empty_like(x)
    rt.native.host_get(y.data_ptr(), 0, a.index, 0, 1 << 20)
    torch.cuda.synchronize()
    assert torch.equal(x, y) and torch.equal(a.local, x)
