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


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (512, 768, 1024), (300, 520, 136), (2048, 2048, 4096)])
def test_gemm_cta_pair_matches_fp32_reference(M, N, K):
    """The cta_group::2 variant (256 x 256 tiles on CTA pairs)."""
    from opengda_b200.ops.gemm import gemm, check_errors
    g = torch.Generator(device="cuda").manual_seed(M + 11 * N + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    C = gemm(A, B, bn=512)
    torch.cuda.synchronize()
    check_errors()
    ref = _ref(A, B)
    err = (C.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-2, err
