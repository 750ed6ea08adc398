"""The persistent command-ring kernel on one GPU: host-queued puts, gets and signals into
this rank's own symmetric buffers (peer == self), in order, plus the idle-timeout exit."""
import time

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


def test_cmdring_puts_gets_signals(rt):
    # Everything is allocated before start() and checked after stop(): no kernel launches
    # while the ring kernel is resident (see the lazy-loading note in CmdRing).
    from opengda_b200 import native
    from opengda_b200.parallel.cmdring import CmdRing
    buf = rt.alloc_tensor((1 << 20,), torch.uint8)
    src = torch.randint(0, 256, (1 << 20,), dtype=torch.uint8, device="cuda")
    back = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    word = rt.signal_alloc(1)
    torch.cuda.synchronize()
    ring = CmdRing(rt, nslots=8)
    ring.start()
    last = 0
    for k in range(64):  # 64 puts through 8 slots: slots are recycled
        off = (k * 12289) % ((1 << 20) - 8192)
        last = ring.put(src.data_ptr() + off, rt.rank, buf.index, off, 1 + (k * 131) % 8192)
    sig = ring.signal(rt.rank, word, 4242)
    got = ring.get(back.data_ptr(), rt.rank, buf.index, 0, 4096)
    ring.wait(got)
    assert sig == last + 1 and got == sig + 1 and ring.completed() == got
    ring.stop()
    assert ring.status() == 0 and not ring.running
    host = buf.local.cpu()
    s = src.cpu()
    for k in range(64):
        off = (k * 12289) % ((1 << 20) - 8192)
        n = 1 + (k * 131) % 8192
        assert torch.equal(host[off:off + n], s[off:off + n]), k
    assert torch.equal(back.cpu(), host[:4096])
    sig_word = native().tensor_from_ptr(rt.signal_local(word), [1], "int64", rt.gpu_id)
    assert int(sig_word.item()) == 4242


def test_cmdring_idle_timeout_exit_and_restart(rt):
    from opengda_b200.parallel.cmdring import CmdRing
    buf = rt.alloc_tensor((4096,), torch.uint8)
    src = torch.full((4096,), 9, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ring = CmdRing(rt, nslots=4, idle_timeout_ms=200)
    ring.start()
    t0 = time.time()
    while ring.status() < 0 and time.time() - t0 < 10:
        time.sleep(0.05)
    assert ring.status() == 1  # GICC_ETIMEDOUT: exited on its own after 200 ms idle
    ring.stop()
    ring.start()  # launches again from the same ring
    ring.wait(ring.put(src.data_ptr(), rt.rank, buf.index, 0, 4096))
    ring.stop()
    assert torch.equal(buf.local.cpu(), src.cpu())
