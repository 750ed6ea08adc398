"""Rank program of the GPU rank-loss test (launched by opengda_b200.parallel.launch with
multicast off): every rank runs a few steps of device work against its neighbours (plain
peer stores + a device barrier); between two steps -- after a synchronize, with none of its
kernels in flight -- the leaving rank exits without a word.  The others learn of it on the
host, at the bootstrap barrier that precedes every step's launches, so no kernel of theirs
ever waits on the departed rank.  Each survivor writes what it saw and exits."""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from opengda_b200 import native  # noqa: E402
from opengda_b200.parallel import Barrier, Bootstrap, Runtime  # noqa: E402


def main():
    out, leaver, leave_after = sys.argv[1], int(sys.argv[2]), int(sys.argv[3])
    boot = Bootstrap.from_env()
    rt = Runtime(boot)
    r, n = rt.rank, rt.size
    assert not rt.multicast_supported or os.environ.get("GICC_DISABLE_NVLS") == "1"
    N = native()
    buf = rt.alloc_tensor((1 << 20,), torch.uint8)
    src = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    bar = Barrier(rt)
    res = {"rank": r, "steps_done": 0, "detected": None}
    for step in range(6):
        try:
            boot.barrier()  # host-side liveness check before any launch of this step
        except Exception as e:  # the departed rank: stop launching, report, leave
            res["detected"] = f"{type(e).__name__}: {e}"
            break
        N.k_fill_pattern(src.data_ptr(), 1 << 20, 10 * step + r)
        N.k_copy(buf.ptr((r + 1) % n), src.data_ptr(), 1 << 20)
        bar.device_barrier()
        torch.cuda.synchronize()  # nothing of this rank is in flight past this point
        rt.check_device_errors()
        res["steps_done"] = step + 1
        if r == leaver and step + 1 == leave_after:
            os._exit(0)  # leaves between steps, without the goodbye handshake
    with open(f"{out}.{r}", "w") as f:
        json.dump(res, f)
    os._exit(0)  # a failed job: skip the collective teardown


if __name__ == "__main__":
    main()
