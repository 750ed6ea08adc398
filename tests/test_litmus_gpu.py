"""Memory-model litmus tests of the flag protocols on a GPU: the two roles run as two CTAs
of one launch (always co-resident), with random delays between the operations."""
import pytest

from opengda_b200.utils import litmus

pytestmark = pytest.mark.gpu


def test_message_passing_release_acquire():
    r = litmus.run(litmus.MP, iters=20000, k=64, max_delay=512)
    assert r["status"] == 0 and r["violations"] == 0, r


def test_store_buffering_with_fence_sc():
    r = litmus.run(litmus.SB, iters=20000, use_fence=True, max_delay=512)
    assert r["status"] == 0, r
    assert r["outcomes"]["00"] == 0, r
    assert sum(r["outcomes"].values()) == 20000


def test_store_buffering_without_fence_completes():
    # (0, 0) is allowed here; the test only checks that the run completes and is counted
    r = litmus.run(litmus.SB, iters=5000, use_fence=False, max_delay=512)
    assert r["status"] == 0 and sum(r["outcomes"].values()) == 5000, r
