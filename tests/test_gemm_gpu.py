"""Numerics of the tcgen05 GEMM against a plain fp32 PyTorch reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(A, B, alpha=1.0):
    return alpha * (A.float() @ B.float().t())


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 256), (200, 384, 136), (1000, 264, 520),
                                   (2048, 2048, 4096), (128, 128, 8192)])
@pytest.mark.parametrize("bn", [256, 128])
def test_gemm_bf16_matches_fp32_reference(M, N, K, bn):
    from opengda_b200.ops.gemm import gemm, check_errors
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    C = gemm(A, B, bn=bn)
    torch.cuda.synchronize()
    check_errors()
    ref = _ref(A, B)
    err = (C.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1e-2 * scale + 1e-2, (err, scale)


def test_gemm_f32_out_and_alpha():
    from opengda_b200.ops.gemm import gemm, check_errors
    torch.manual_seed(0)
    A = torch.randn(384, 1024, device="cuda").to(torch.bfloat16)
    B = torch.randn(512, 1024, device="cuda").to(torch.bfloat16)
    C = gemm(A, B, alpha=0.5, out_dtype=torch.float32)
    torch.cuda.synchronize()
    check_errors()
    ref = _ref(A, B, 0.5)
    torch.testing.assert_close(C, ref, rtol=1e-4, atol=1e-3)


def test_gemm_strided_views():
    from opengda_b200.ops.gemm import gemm, check_errors
    torch.manual_seed(1)
    Abig = torch.randn(512, 2048, device="cuda").to(torch.bfloat16)
    Bbig = torch.randn(768, 2048, device="cuda").to(torch.bfloat16)
    A = Abig[:, 512:1536]
    B = Bbig[256:, 512:1536]
    C = gemm(A, B)
    torch.cuda.synchronize()
    check_errors()
    ref = _ref(A, B)
    assert (C.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (512, 768, 1024), (300, 520, 136), (2048, 2048, 4096),
                                   (4352, 1800, 200)])
@pytest.mark.parametrize("bn", [512, 1024])
def test_gemm_cta_pair_matches_fp32_reference(M, N, K, bn):
    """The cta_group::2 variants: 256 x 256 tiles (bn=512) and 256 x 512 tiles with one
    512-column TMEM accumulator drained by 8 epilogue warps (bn=1024); ragged M, N and K
    edges included, and more tiles than CTA pairs (4352 x 1800: 17 x 4 wide tiles)."""
    from opengda_b200.ops.gemm import gemm, check_errors
    g = torch.Generator(device="cuda").manual_seed(M + 11 * N + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    C = gemm(A, B, bn=bn)
    torch.cuda.synchronize()
    check_errors()
    ref = _ref(A, B)
    err = (C.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-2, err


@pytest.mark.parametrize("l2_hint,prefetch", [(1, 0), (2, 0), (0, 2), (0, 8), (1, 4)])
def test_gemm_cta_pair_load_options(l2_hint, prefetch):
    """The CTA-pair kernel's L2 eviction hints and L2 prefetch distance change only how the
    operands are loaded: results equal the fp32 reference (prefetch past the last k-step of a
    tile is skipped; 4352 x 1800 x 1000 has ragged edges and 16 k-steps per tile)."""
    from opengda_b200.ops.gemm import gemm, check_errors, set_tuning, tuning
    g = torch.Generator(device="cuda").manual_seed(l2_hint * 10 + prefetch)
    A = torch.randn(4352, 1000, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(1800, 1000, device="cuda", generator=g).to(torch.bfloat16)
    base = tuning()
    try:
        set_tuning(**dict(base, pair_l2_hint=l2_hint, pair_prefetch=prefetch))
        for bn in (512, 1024):
            C = gemm(A, B, bn=bn)
            torch.cuda.synchronize()
            check_errors()
            ref = _ref(A, B)
            err = (C.float() - ref).abs().max().item()
            assert err <= 1e-2 * ref.abs().max().item() + 1e-2, (bn, err)
    finally:
        set_tuning(**base)


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (300, 520, 200), (1000, 264, 516), (2048, 2048, 4096)])
@pytest.mark.parametrize("bn", [256, 512, 1024])
def test_gemm_fp32_on_tensor_cores_matches_fp64(M, N, K, bn):
    """fp32 GEMM from three tf32 products on the tensor cores (one CTA, or CTA pairs with
    256 x 256 / 256 x 512 tiles), against an fp64 product: the error per element stays below
    1e-5 of sum |A||B| (fp32 FMA itself is near 6e-8 per term); ragged M, N and K' = 3K not a
    multiple of the 32-element k-block included."""
    from opengda_b200.ops.gemm import gemm_fp32, check_errors
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(N, K, device="cuda", generator=g)
    C = gemm_fp32(A, B, alpha=0.5, bn=bn)
    torch.cuda.synchronize()
    check_errors()
    ref = 0.5 * (A.double() @ B.double().t())
    scale = 0.5 * (A.double().abs() @ B.double().abs().t())
    err = float(((C.double() - ref).abs() / scale).max())
    assert err < 1e-5, err


@pytest.mark.parametrize("N", [100, 264])
@pytest.mark.parametrize("bn", [128, 256, 512, 1024])
@pytest.mark.parametrize("out_f32", [False, True])
def test_gemm_unaligned_out_and_ragged_n(N, bn, out_f32):
    """C views whose base is not 16-byte aligned, and N not a multiple of the 16-byte vector
    (8 bf16 / 4 f32 columns): every element of C is stored (element stores where vector
    stores do not fit) and nothing outside it."""
    from opengda_b200.ops.gemm import gemm, check_errors
    M, K = 300, 136
    g = torch.Generator(device="cuda").manual_seed(N + bn)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    dt = torch.float32 if out_f32 else torch.bfloat16
    ref = _ref(A, B, 0.5)
    big = torch.full((M + 1, N + 8), 7.0, device="cuda", dtype=dt)
    for off in (0, 3):
        C = big[:M, off:off + N]
        out = gemm(A, B, out=C, alpha=0.5, out_dtype=dt, bn=bn)
        torch.cuda.synchronize()
        check_errors()
        err = (out.float() - ref).abs().max().item()
        assert err <= 1e-2 * ref.abs().max().item() + 1e-2, (off, err)
    assert (big[M] == 7.0).all() and (big[:M, N + 3:] == 7.0).all()


@pytest.mark.parametrize("M,N,K", [(4352, 1800, 1000), (300, 520, 136), (256, 256, 64), (2048, 2048, 4096),
                                   (300, 100, 136)])
@pytest.mark.parametrize("tma", [1, 0])
def test_gemm_cta_pair_store_paths(M, N, K, tma):
    """bf16 C stored by the pair kernels in 32 x 32 boxes through shared memory and TMA (the
    default) or per thread: ragged M and N (partial boxes clipped, boxes past the edge
    skipped), alpha, and a C view whose base is not 16-byte aligned (per-thread stores)."""
    from opengda_b200.ops.gemm import gemm, check_errors, set_tuning, tuning
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    ref = _ref(A, B, 0.5)
    base = tuning()
    try:
        set_tuning(**dict(base, pair_tma_store=tma))
        for bn in (512, 1024):
            big = torch.full((M + 1, N + 40), 7.0, device="cuda", dtype=torch.bfloat16)
            for C in (big[:M, :N], big[:M, 3:N + 3]):  # 16-byte pitch; unaligned base -> fallback
                out = gemm(A, B, out=C, alpha=0.5, bn=bn)
                torch.cuda.synchronize()
                check_errors()
                err = (out.float() - ref).abs().max().item()
                assert err <= 1e-2 * ref.abs().max().item() + 1e-2, (bn, err)
            assert (big[M] == 7.0).all() and (big[:M, N + 3:] == 7.0).all()  # nothing stored past C
    finally:
        set_tuning(**base)


@pytest.mark.gpu
@pytest.mark.parametrize("skew_ns", [0, 20000])
def test_gemm_core_publishes_each_tile_once_after_all_epilogue_warps(skew_ns):
    """The hook that the distributed epilogues use to publish a finished tile (a flag or a
    counter on the owner GPU) must run once per tile and only after all four epilogue warps
    are done with it, also when one warp lags behind the others."""
    from opengda_b200 import native

    torch.manual_seed(0)
    M, N, K = 128 * 148 * 3, 512, 128  # 3 tiles per CTA in each accumulator parity
    A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    B = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    tiles = (M // 128) * (N // 256)
    counters = torch.zeros(2 * tiles + 1, dtype=torch.int32, device="cuda")
    native().gemm_tile_done_selftest(A, B, counters, skew_ns)
    torch.cuda.synchronize()
    assert int(counters[2 * tiles]) == 0
    assert torch.equal(counters[:tiles], torch.full((tiles,), 4, dtype=torch.int32, device="cuda"))
    assert torch.equal(counters[tiles:2 * tiles], torch.ones(tiles, dtype=torch.int32, device="cuda"))
