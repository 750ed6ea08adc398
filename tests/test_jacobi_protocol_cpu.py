"""The synchronisation protocol of the persistent Jacobi kernel (k_jacobi_persistent),
restated on CPU and run by a randomised scheduler over several ranks and CTAs.

Model: CTA c of rank q owns rows [lo, hi) of its rank's rows (contiguous blocks of
ceil(rows / G)); an iteration of a CTA reads rows lo-1 .. hi of the read buffer and writes
rows lo .. hi-1 of the other, and the owners of row 1 / row `rows` push it into the
neighbour rank's halo row of that buffer and add one arrival per column chunk.  Before
iteration gi a CTA waits for its neighbouring CTAs' done counters (>= gi, from the second
iteration of a launch on) and, at the ends, for the halo arrivals (>= gi * chunks).  The
scheduler runs any enabled CTA-iteration; the checks: the run never blocks, every read sees
the previous iteration's data, and no row is overwritten while an earlier iteration still
has to read it."""
import random

import pytest


def _blocks(rows, G):
    per = (rows + G - 1) // G
    return [(min(1 + c * per, rows + 1), min(1 + (c + 1) * per, rows + 1)) for c in range(G)]


def _simulate(rows_per_rank, G, iters, chunks, seed):
    rng = random.Random(seed)
    n = len(rows_per_rank)
    blocks = [_blocks(R, G) for R in rows_per_rank]
    # ver[q][p][x]: field version held by row x of buffer p (0 = initial, in both buffers)
    ver = [[[0] * (R + 2) for _ in range(2)] for R in rows_per_rank]
    done = [[0] * G for _ in range(n)]
    top_flag, bot_flag = [0] * n, [0] * n
    it = [[0] * G for _ in range(n)]
    total = n * G * iters
    steps = 0
    while steps < total:
        ready = []
        for q in range(n):
            R = rows_per_rank[q]
            for c in range(G):
                gi = it[q][c]
                if gi == iters:
                    continue
                lo, hi = blocks[q][c]
                own_top, own_bot = lo == 1 and lo < hi, lo <= R < hi
                if gi > 0 and ((c > 0 and done[q][c - 1] < gi) or (c + 1 < G and done[q][c + 1] < gi)):
                    continue
                if own_top and q > 0 and top_flag[q] < gi * chunks:
                    continue
                if own_bot and q < n - 1 and bot_flag[q] < gi * chunks:
                    continue
                ready.append((q, c))
        assert ready, ("blocked", it, done, top_flag, bot_flag)
        q, c = rng.choice(ready)
        R = rows_per_rank[q]
        gi = it[q][c]
        rd, wr = gi & 1, (gi & 1) ^ 1
        lo, hi = blocks[q][c]
        own_top, own_bot = lo == 1 and lo < hi, lo <= R < hi
        if lo < hi:
            for x in range(lo - 1, hi + 1):
                if (x == 0 and q == 0) or (x == R + 1 and q == n - 1):
                    continue  # the global boundary rows are constant
                assert ver[q][rd][x] == gi, (q, c, gi, x, ver[q][rd][x])
            for x in range(lo, hi):
                # every CTA that reads row x (its block or an adjacent one) finished gi-1
                for c2, (l2, h2) in enumerate(blocks[q]):
                    if l2 < h2 and l2 - 1 <= x <= h2:
                        assert c2 == c or done[q][c2] >= gi, ("overwrite before read", q, c, gi, x, c2)
                ver[q][wr][x] = gi + 1
            if own_top and q > 0:  # row 1 -> upper rank's bottom halo of its buffer wr
                up = rows_per_rank[q - 1]
                reader = next(c2 for c2, (l2, h2) in enumerate(blocks[q - 1]) if l2 <= up < h2)
                assert done[q - 1][reader] >= gi, ("halo overwritten before its reader finished", q, gi)
                assert ver[q - 1][wr][up + 1] == gi - 1 or gi == 0, ("halo overwrite", q, gi)
                ver[q - 1][wr][up + 1] = gi + 1
                bot_flag[q - 1] += chunks
            if own_bot and q < n - 1:  # row R -> lower rank's top halo of its buffer wr
                reader = next(c2 for c2, (l2, h2) in enumerate(blocks[q + 1]) if l2 == 1 and l2 < h2)
                assert done[q + 1][reader] >= gi, ("halo overwritten before its reader finished", q, gi)
                assert ver[q + 1][wr][0] == gi - 1 or gi == 0, ("halo overwrite", q, gi)
                ver[q + 1][wr][0] = gi + 1
                top_flag[q + 1] += chunks
        done[q][c] = gi + 1
        it[q][c] += 1
        steps += 1
    # halo rows of the global boundary never change; every owned row reached the last version
    for q in range(n):
        for x in range(1, rows_per_rank[q] + 1):
            assert ver[q][iters & 1][x] == iters


@pytest.mark.parametrize("rows_per_rank,G", [([40], 7), ([10, 11], 4), ([9, 9, 8], 3), ([5, 6, 5, 6], 8),
                                             ([33, 32], 5)])
@pytest.mark.parametrize("seed", range(4))
def test_persistent_jacobi_protocol(rows_per_rank, G, seed):
    _simulate(rows_per_rank, G, iters=6, chunks=3, seed=seed)
