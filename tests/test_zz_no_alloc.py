"""The allocation-free entry point gicc_jacobi_step_norm_noalloc, called through its
exported C symbol, against the library's regular Jacobi entry point (which takes its norm
accumulator from the caller).  Some callers cannot allocate device memory when they call
into the library -- code inside an allocator or an out-of-memory path, or an embedder whose
memory manager owns every allocation -- so this entry point keeps its working memory in a
static device array.  Collected last (file name) so a failure here comes after every other
test has run."""
import ctypes
import os

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "opengda_b200", "lib", "libgicc.so")

pytestmark = pytest.mark.gpu


def _entry():
    from opengda_b200 import native  # loads torch, the binding and libgicc.so

    native()
    lib = ctypes.CDLL(LIB)
    fn = lib.gicc_jacobi_step_norm_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    return fn


@pytest.mark.parametrize("nx, ny", [(2048, 1030), (2052, 37)])
def test_noalloc_jacobi_matches_regular_entry_point_twice(nx, ny):
    """nx = 2048 fills every lane of every block; nx = 2052 (not a multiple of the 128
    columns a warp covers) leaves most lanes of the last block idle, and ny = 37 leaves the
    last row block short."""
    from opengda_b200 import native

    fn = _entry()
    n = native()
    rows = ny - 2
    a = torch.empty(rows + 2, nx, dtype=torch.float32, device="cuda")
    n.k_jacobi_init(a.data_ptr(), 0, nx, ny, rows, 1, 3)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row: the shared array keeps the last call's contents
        b_ref = a.clone()
        norm_ref = torch.zeros(1, dtype=torch.float64, device="cuda")
        n.k_jacobi_step(a.data_ptr(), b_ref.data_ptr(), nx, rows, 0, 0, 0, 0, 0, 0, 0, 0, norm_ref.data_ptr(), 0, 0)
        b = a.clone()
        norm = torch.full((1,), -1.0, dtype=torch.float64, device="cuda")
        rc = fn(a.data_ptr(), b.data_ptr(), nx, rows, norm.data_ptr(), stream)
        torch.cuda.synchronize()
        assert rc == 0, call
        assert torch.equal(b, b_ref), call
        ref = float(norm_ref.item())
        assert ref > 0 and abs(float(norm.item()) - ref) <= 1e-5 * ref, (call, float(norm.item()), ref)
        a = b


def test_noalloc_rejects_oversized_grid():
    fn = _entry()
    a = torch.zeros(16, dtype=torch.float32, device="cuda")
    norm = torch.zeros(1, dtype=torch.float64, device="cuda")
    # 65536 columns x 32768 rows needs 64 x 2048 = 131072 partial sums > 65536
    rc = fn(a.data_ptr(), a.data_ptr(), 65536, 32768, norm.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 1  # cudaErrorInvalidValue, nothing launched
    # input and output must not overlap (the sweep would read cells it already rewrote)
    f = torch.zeros(10 * 64, dtype=torch.float32, device="cuda")
    rc = fn(f.data_ptr(), f.data_ptr(), 64, 8, norm.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    torch.cuda.synchronize()
