"""Host logic of the ring-stripe matmul (opengda_b200.models.ring_mm), on CPU: the per-step
plan every rank follows (which stripe it holds, which landing buffer it reads and fills, and
the counter values it waits for) is run by a randomised scheduler of n ranks that executes
steps in any order the waits allow.  The run must never block, every rank must see the
stripe of rank (r - s) mod n in step s, and no landing buffer may be overwritten before the
step that reads it has finished."""
import random

import pytest

from opengda_b200.models.ring_mm import ring_step_plan


def _simulate(n, calls, push_ctas, seed):
    rng = random.Random(seed)
    grid = push_ctas + 5
    arrivals, consumed = [0] * n, [0] * n
    land = [[None, None] for _ in range(n)]     # stripe id in each landing buffer
    pending = [[False, False] for _ in range(n)]  # written and not yet read
    pc = [0] * n                                # steps done by each rank
    total = calls * n
    while any(p < total for p in pc):
        ready = []
        for r in range(n):
            if pc[r] == total:
                continue
            call, s = pc[r] // n + 1, pc[r] % n
            p = ring_step_plan(n, r, call, s, push_ctas, pc[r], grid)
            if p["arrivals_target"] is not None and arrivals[r] < p["arrivals_target"]:
                continue
            if p["push"] is not None and consumed[r] < p["consumed_target"]:
                continue
            ready.append((r, p))
        assert ready, ("blocked", pc, arrivals, consumed)
        r, p = rng.choice(ready)
        right, left = (r + 1) % n, (r - 1) % n
        if p["read"] is None:
            held = r
        else:
            assert pending[r][p["read"]], (r, pc[r], "reads a buffer nobody filled")
            held = land[r][p["read"]]
            pending[r][p["read"]] = False
        assert held == p["col_block"] == (r - pc[r] % n) % n, (r, pc[r], held, p)
        if p["push"] is not None:
            assert not pending[right][p["push"]], (r, pc[r], "overwrites a stripe not yet read")
            land[right][p["push"]] = held
            pending[right][p["push"]] = True
            arrivals[right] += push_ctas
        assert p["ticket_target"] == (pc[r] + 1) * grid
        consumed[left] += 1
        pc[r] += 1
    assert arrivals == [calls * (n - 1) * push_ctas] * n and consumed == [calls * n] * n


@pytest.mark.parametrize("n", [2, 3, 4, 8])
@pytest.mark.parametrize("seed", range(5))
def test_ring_plan_never_blocks_and_never_overwrites(n, seed):
    _simulate(n, calls=4, push_ctas=3, seed=seed)


def test_ring_plan_single_rank():
    p = ring_step_plan(1, 0, 7, 0, 0, 6, 16)
    assert p["read"] is None and p["push"] is None and p["arrivals_target"] is None and p["col_block"] == 0


def test_ring_matmul_shape_checks():
    from opengda_b200.models.ring_mm import RingMatmul
    with pytest.raises(ValueError):
        RingMatmul(100)        # N / ranks not a multiple of 64
    with pytest.raises(ValueError):
        RingMatmul(64 * 3 + 8)
