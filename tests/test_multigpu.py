"""Multi-GPU tests: one process per GPU (2..8 ranks), NVLink puts/gets, host-queued puts,
barriers, allreduce and both distributed GEMM modes, each checked against a reference."""
import json
import os
import sys

import pytest

from opengda_b200.parallel.launch import launch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
WORKER = os.path.join(os.path.dirname(__file__), "workers", "gpu_worker.py")


def test_multigpu_suite(tmp_path):
    import torch
    n = min(torch.cuda.device_count(), 8)
    out = str(tmp_path / "mg")
    rc = launch(n, [sys.executable, WORKER, out], timeout=600,
                extra_env={"GICC_TIMEOUT_MS": "5000", "GICC_BOOTSTRAP_TIMEOUT_MS": "120000"})
    res = [json.load(open(f"{out}.{r}")) for r in range(n)]
    assert rc == 0, res
    for r in res:
        assert r["put_bad_bytes"] == 0 and r["get_bad_bytes"] == 0 and r["queued_bad_bytes"] == 0, r
        assert r["single_flag"] == 42 and r["continuous_count"] == 10000, r
        for k, v in r["allreduce_maxerr"].items():
            assert v < 0.05 * n, (k, v)
        for k in ("gemm_ag_relerr", "gemm_rs_relerr", "gemm_ag_fused_relerr", "gemm_rs_fused_relerr"):
            assert r[k] < 1e-2, (k, r)
        assert r["jacobi_mismatch"] == 0, r
        assert r["moe_relerr"] < 2e-2, r
        assert r["am_counter_ok"] and r["am_checksum_ok"], r
    assert all(r["context_ok_after_inject"] for r in res), res
    timed_out = [r["rank"] for r in res if r["inject_error"]["status"] == "ETIMEDOUT"]
    assert timed_out and all(res[i]["inject_error"]["where"] == "barrier" for i in timed_out), res
    mp, sb = res[0]["litmus_mp"], res[0]["litmus_sb"]
    assert mp["status"] == 0 and mp["violations"] == 0, mp
    assert sb["status"] == 0 and sb["outcomes"]["00"] == 0 and sum(sb["outcomes"].values()) == 20000, sb
    print(json.dumps(res))
