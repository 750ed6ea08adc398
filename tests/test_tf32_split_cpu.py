"""The fp32-on-tensor-cores method (ops.gemm.gemm_fp32, the ring matmul's default mode),
restated on the CPU: x = hi + lo with hi = x rounded to tf32 (nearest, ties away, as
cvt.rna.tf32.f32) and lo the exact remainder; A.B^T ~ Ahi.Bhi + Ahi.Blo + Alo.Bhi with the
MMA reading lo as tf32 too.  The error per element stays near 2^-21 of sum |a b| -- the bound
the GPU tests hold the kernels to (1e-5)."""
import numpy as np
import pytest


def to_tf32_rna(x: np.ndarray) -> np.ndarray:
    """Round fp32 to tf32 (10 explicit mantissa bits), nearest with ties away from zero."""
    b = x.astype(np.float32).view(np.uint32)
    r = ((b + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).astype(np.uint32)
    return r.view(np.float32)


def to_tf32_trunc(x: np.ndarray) -> np.ndarray:
    return (x.astype(np.float32).view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


def test_split_is_exact_and_small():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(100000) * np.exp(rng.uniform(-20, 20, 100000))).astype(np.float32)
    hi = to_tf32_rna(x)
    lo = (x - hi).astype(np.float32)
    assert np.array_equal((hi.astype(np.float64) + lo.astype(np.float64)), x.astype(np.float64))  # exact
    assert np.all(hi.view(np.uint32) & np.uint32(0x1FFF) == 0)  # hi is a tf32 value
    assert np.all(np.abs(lo) <= np.abs(x) * 2.0 ** -11 * (1 + 2.0 ** -10))


@pytest.mark.parametrize("lo_in_mma", [to_tf32_trunc, to_tf32_rna])
def test_three_products_error_bound(lo_in_mma):
    rng = np.random.default_rng(1)
    M, N, K = 64, 48, 1536
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    Ah, Bh = to_tf32_rna(A), to_tf32_rna(B)
    Al, Bl = lo_in_mma((A - Ah).astype(np.float32)), lo_in_mma((B - Bh).astype(np.float32))
    # K' = 3K operands as laid out for the GEMM: (hi, hi, lo) . (hi, lo, hi)
    Ap = np.concatenate([Ah, Ah, Al], axis=1).astype(np.float64)
    Bp = np.concatenate([Bh, Bl, Bh], axis=1).astype(np.float64)
    C = Ap @ Bp.T  # products of tf32 values are exact in fp64; accumulation error not modelled
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    scale = np.abs(A.astype(np.float64)) @ np.abs(B.astype(np.float64)).T
    err = np.max(np.abs(C - ref) / scale)
    assert err < 2.0 ** -20, err
    # one tf32 product alone is far worse: the split is what buys fp32-level accuracy
    one = (Ah.astype(np.float64) @ Bh.astype(np.float64).T)
    err_one = np.max(np.abs(one - ref) / scale)
    assert err_one > 1e-5 and err_one > 20 * err, (err_one, err)
