"""Jacobi: the CPU oracle on its own (CPU) and the fused kernel against it (GPU)."""
import numpy as np
import pytest
import torch

from opengda_b200.models.jacobi import init_field_np, jacobi_np, split_rows


def test_split_rows_covers_interior_unevenly():
    ny = 4099
    for w in (1, 2, 3, 8):
        parts = [split_rows(ny, w, r) for r in range(w)]
        assert sum(p[0] for p in parts) == ny - 2
        assert parts[0][1] == 1
        for r in range(1, w):
            assert parts[r][1] == parts[r - 1][1] + parts[r - 1][0]


def test_oracle_boundary_and_fixed_point():
    a = init_field_np(16, 12)
    assert (a[0] == 1).all() and (a[-1] == 0).all() and (a[1:-1, 0] == 0).all()
    assert ((a[1:-1, 1:-1] >= 0) & (a[1:-1, 1:-1] < 1)).all()
    b = jacobi_np(16, 12, 5000)
    # converges to the harmonic solution: monotone decay away from the hot edge
    assert b[1, 8] > b[5, 8] > b[10, 8] >= 0


@pytest.mark.gpu
@pytest.mark.parametrize("nx,ny,iters", [(256, 130, 7), (1028, 67, 20), (4096, 40, 3)])
def test_jacobi_kernel_bit_exact_vs_oracle(nx, ny, iters):
    from opengda_b200.models.jacobi import Jacobi
    from opengda_b200.ops.gemm import check_errors
    j = Jacobi(nx, ny)
    init = j.owned().cpu().numpy()
    np.testing.assert_array_equal(init, init_field_np(nx, ny)[1:-1])
    j.run(iters)
    torch.cuda.synchronize()
    check_errors()
    ref = jacobi_np(nx, ny, iters)[1:-1]
    np.testing.assert_array_equal(j.owned().cpu().numpy(), ref)


@pytest.mark.gpu
def test_jacobi_norm():
    from opengda_b200.models.jacobi import Jacobi
    j = Jacobi(512, 66)
    j.run(4)
    prev = j.owned().cpu().numpy().copy()
    nrm = j.run(1, norm_last=True)
    cur = j.owned().cpu().numpy()
    ref = float(np.sqrt(((cur.astype(np.float64) - prev) ** 2).sum()))
    assert abs(nrm - ref) <= 1e-5 * max(ref, 1.0)
