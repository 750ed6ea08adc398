"""CPU rank for the protocol tests: maps a shared file and runs the barrier / active-message
protocols (the kernels' code, compiled for the host) against the other ranks."""
import mmap
import os
import sys
import ctypes

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from opengda_b200 import native  # noqa: E402


def main():
    path, what, out = sys.argv[1], sys.argv[2], sys.argv[3]
    args = [int(x) for x in sys.argv[4:]]
    rank, size = int(os.environ["GICC_RANK"]), int(os.environ["GICC_SIZE"])
    fd = os.open(path, os.O_RDWR)
    mm = mmap.mmap(fd, os.fstat(fd).st_size)
    addr = ctypes.addressof(ctypes.c_char.from_buffer(mm))
    n = native()
    if what == "barrier":
        iters, mode, skip_rank = args
        skip_at = iters // 2 if rank == skip_rank else -1
        st, fail = n.cpu_barrier_run(addr, rank, size, iters, mode, 10_000_000_000, skip_at)  # ranks start seconds apart
        res = f"{st} {fail}"
    elif what == "am":
        nslots, nmsg, nreq = args
        st, c, k = n.cpu_am_run(addr, rank, size, nslots, nmsg, nreq, 20_000_000_000)
        res = f"{st} {c} {k}"
    elif what == "am_drop":
        # rank 0 waits for a message from rank 1, which never sends it
        res = str(n.cpu_am_wait_one(addr, rank, size, 4, 1, 300_000_000)) if rank == 0 else "idle"
    elif what == "barrier_inject":
        iters, mode, inj_rank, inj_mode, inj_at = args
        st, fail = n.cpu_barrier_run_inject(addr, rank, size, iters, mode, 10_000_000_000,
                                            inj_mode if rank == inj_rank else 0, inj_at)
        res = f"{st} {fail}"
    elif what == "litmus":
        test, iters, k, fence, max_delay = args
        st, v = n.cpu_litmus_run(addr, rank, test, iters, k, fence, 7, max_delay, 20_000_000_000)
        res = f"{st} {v}"
    with open(f"{out}.{rank}", "w") as f:
        f.write(res)
    del addr
    mm.close()
    os.close(fd)


if __name__ == "__main__":
    main()
