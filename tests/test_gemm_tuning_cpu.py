"""The GEMM tuning knobs (raster group, L2 hints) are validated and restored on the host."""
import pytest

from opengda_b200.ops.gemm import set_tuning, tuning


def test_tuning_roundtrip_and_validation():
    default = {"group_m": 16, "l2_hint": 0, "pair_group_m": 16, "pair_l2_hint": 0, "pair_prefetch": 0,
               "pair_tma_store": 1}
    assert tuning() == default
    custom = {"group_m": 8, "l2_hint": 2, "pair_group_m": 4, "pair_l2_hint": 1, "pair_prefetch": 6,
              "pair_tma_store": 0}
    try:
        set_tuning(**custom)
        assert tuning() == custom
        for bad in ({"group_m": 0}, {"l2_hint": 3}, {"l2_hint": -1}, {"pair_group_m": 0}, {"pair_l2_hint": 3},
                    {"pair_prefetch": -1}, {"pair_prefetch": 65}, {"pair_tma_store": 2}):
            with pytest.raises(RuntimeError):
                set_tuning(**bad)
        assert tuning() == custom  # a rejected call changes nothing
    finally:
        set_tuning()
    assert tuning() == default


def test_tuning_from_environment():
    import os
    import subprocess
    import sys
    code = "from opengda_b200.ops.gemm import tuning; print(tuning())"
    env = dict(os.environ, GICC_GEMM_GROUP_M="8", GICC_GEMM_L2_HINT="1", GICC_GEMM_PAIR_PREFETCH="4")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert "'group_m': 8" in out.stdout and "'l2_hint': 1" in out.stdout, out.stdout + out.stderr
    assert "'pair_prefetch': 4" in out.stdout, out.stdout + out.stderr
    env["GICC_GEMM_L2_HINT"] = "5"
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode != 0 and "GICC_GEMM_L2_HINT" in out.stderr
