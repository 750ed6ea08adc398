"""The CTA-pair core's k-step bookkeeping with the half-0 lag (gemm_core2.cuh, NH = 2),
restated on the host: for each tile the MMA thread first waits on the "full" barriers of
`lag` = min(nk, S - 1) stages with the parity phase ^ (stage + i >= S), issues half 0 there,
and after the epilogue frees half 1 issues half 1 of the same k-steps while advancing
stage/phase; then the remaining k-steps in order.  Every (stage, parity) it waits on must be
the producer's next fill, in the same order, and every fill must be released once, across
tiles of any length."""
import pytest


def producer_fills(nks, S):
    stage, phase, out = 0, 0, []
    for nk in nks:
        for _ in range(nk):
            out.append((stage, phase))
            stage += 1
            if stage == S:
                stage, phase = 0, phase ^ 1
    return out


def mma_waits_and_releases(nks, S, lag_on=True):
    stage, phase = 0, 0
    waits, releases = [], []
    for nk in nks:
        lag = min(nk, S - 1) if lag_on else 0
        for i in range(lag):  # half 0 of the first `lag` k-steps, stages held
            st = (stage + i) % S
            waits.append((st, phase ^ (1 if stage + i >= S else 0)))
        for i in range(lag):  # half 1 catches up; the stages go back in order
            releases.append((stage, phase))
            stage += 1
            if stage == S:
                stage, phase = 0, phase ^ 1
        for _ in range(lag, nk):
            waits.append((stage, phase))
            releases.append((stage, phase))
            stage += 1
            if stage == S:
                stage, phase = 0, phase ^ 1
    return waits, releases


@pytest.mark.parametrize("S", [4, 6])
@pytest.mark.parametrize("nks", [[1, 1, 1, 1, 1], [2, 3, 1, 5], [3] * 7, [128, 128, 2, 4, 9], [5, 1, 7, 3, 3, 2, 11]])
def test_lag_waits_match_producer_fills(S, nks):
    fills = producer_fills(nks, S)
    waits, releases = mma_waits_and_releases(nks, S)
    assert waits == fills
    assert releases == fills
    assert mma_waits_and_releases(nks, S, lag_on=False) == (fills, fills)

