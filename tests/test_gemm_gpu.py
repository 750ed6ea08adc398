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
