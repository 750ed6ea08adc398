"""Rank program for the bootstrap tests (launched by opengda_b200.parallel.launch)."""
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from opengda_b200.parallel.bootstrap import Bootstrap, allreduce_max, allreduce_min, allreduce_sum  # noqa: E402


def main():
    mode = sys.argv[1]
    out = sys.argv[2]
    b = Bootstrap.from_env()
    r, n = b.rank(), b.size()
    res = []
    if mode == "collectives":
        assert b.local_size() == n and b.local_rank() == r
        assert all(b.locality_map())
        g = b.allgather(bytes([r]) * (r + 1))
        assert g == [bytes([q]) * (q + 1) for q in range(n)], g
        root = n - 1
        v = b.broadcast(b"hello-from-root" if r == root else None, root=root)
        assert v == b"hello-from-root"
        assert b.broadcast_obj({"x": r} if r == 0 else None) == {"x": 0}
        # ring sendrecv (reference mm ring: send right, receive left)
        got = b.sendrecv(r.to_bytes(4, "little") * 3, (r + 1) % n, 12, (r - 1) % n, tag=7)
        assert got == ((r - 1) % n).to_bytes(4, "little") * 3
        for i in range(20):  # many barriers + ordered p2p streams
            b.barrier()
            if r == 0:
                for q in range(1, n):
                    b.send(i.to_bytes(8, "little"), q, tag=1)
            else:
                assert int.from_bytes(b.recv(8, 0, tag=1), "little") == i
        assert allreduce_sum(b, float(r)) == sum(range(n))
        assert allreduce_min(b, float(r)) == 0
        assert allreduce_max(b, float(r)) == n - 1
        assert b.allgather_fixed("q", r * 10) == [q * 10 for q in range(n)]
        res.append("ok")
    elif mode == "fds":
        # pass a pipe's read end to the next rank; it reads what we wrote
        rfd, wfd = os.pipe()
        os.write(wfd, f"rank{r}".encode())
        os.close(wfd)
        b.native.send_fds((r + 1) % n, 5, [rfd])
        fds = b.native.recv_fds((r - 1) % n, 5, 1)
        data = os.read(fds[0], 64).decode()
        os.close(fds[0])
        os.close(rfd)
        assert data == f"rank{(r - 1) % n}", data
        b.barrier()
        res.append("ok")
    elif mode in ("die", "kill"):
        # rank 1 leaves without saying goodbye (exits, or is killed with SIGKILL); the others
        # must learn it at their barrier
        b.barrier()
        if r == 1:
            if mode == "kill":
                import signal
                os.kill(os.getpid(), signal.SIGKILL)
            os._exit(0)
        t0 = time.time()
        try:
            b.barrier()
            res.append("no-error")
        except Exception as e:  # BootstrapError
            res.append(f"err:{type(e).__name__}:{e}:{time.time() - t0:.2f}")
    elif mode == "abort":
        b.barrier()
        if r == 1:
            b.abort(3, "injected failure")
        t0 = time.time()
        try:
            b.barrier()
            b.barrier()
            res.append("no-error")
        except Exception as e:
            res.append(f"err:{type(e).__name__}:{e}:{time.time() - t0:.2f}")
    elif mode == "timeout":
        b.barrier()
        if r == 1:
            time.sleep(4.0)  # never joins the next barrier in time
            res.append("slept")
        else:
            t0 = time.time()
            try:
                b.barrier()
                res.append("no-error")
            except Exception as e:
                res.append(f"err:{type(e).__name__}:{e}:{time.time() - t0:.2f}")
    elif mode in ("exchange_count", "exchange_kind", "exchange_ok"):
        # the buffer tables exchange() compares before any handle is passed: rank 1 registered
        # one buffer more, or one of another kind; every rank must see the mismatch
        from opengda_b200 import native
        kinds, mc = [0, 0, 1], [0, 1, 0]
        if r == 1 and mode == "exchange_count":
            kinds, mc = kinds + [0], mc + [0]
        if r == 1 and mode == "exchange_kind":
            kinds = [0, 1, 1]
        try:
            native().check_exchange_consistency(b.native, kinds, mc)
            b.barrier()
            res.append("ok")
        except Exception as e:
            res.append(f"err:{type(e).__name__}:{e}")
    with open(f"{out}.{r}", "w") as f:
        f.write("\n".join(res))
    if mode in ("die", "kill", "abort", "timeout", "exchange_count", "exchange_kind"):
        os._exit(0)  # skip the goodbye handshake of a failed job


if __name__ == "__main__":
    main()
