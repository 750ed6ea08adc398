"""MoE layer: routing kernel and the full fused forward (one GPU: every expert local)
against an fp32 PyTorch reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_route_matches_torch_softmax_topk():
    from opengda_b200 import native
    T, E, k = 300, 256, 8
    g = torch.Generator(device="cuda").manual_seed(4)
    logits = torch.randn(T, E, generator=g, device="cuda")
    idx = torch.empty(T * k, dtype=torch.int32, device="cuda")
    w = torch.empty(T * k, dtype=torch.float32, device="cuda")
    counts = torch.empty(E, dtype=torch.int32, device="cuda")
    native().k_moe_route(logits.data_ptr(), T, E, k, idx.data_ptr(), w.data_ptr(), counts.data_ptr())
    torch.cuda.synchronize()
    pw, pi = torch.topk(torch.softmax(logits, -1), k, dim=-1)
    assert torch.equal(idx.view(T, k).long(), pi)
    torch.testing.assert_close(w.view(T, k), pw, rtol=1e-5, atol=1e-6)
    assert torch.equal(counts.long(), torch.bincount(pi.flatten(), minlength=E))


@pytest.mark.parametrize("T,H,E,k,I", [(256, 512, 16, 4, 256), (512, 1024, 32, 8, 512)])
def test_moe_forward_single_gpu(T, H, E, k, I):
    from opengda_b200.models.moe import MoELayer, make_inputs, reference_moe
    from opengda_b200.ops.gemm import check_errors
    layer = MoELayer(T, H, E, k, I, rt=None, weight_std=0.05)
    for call in range(3):  # repeated calls: epochs, cumulative counters, buffer parity
        x, logits = make_inputs(T, H, E, 0, seed=10 + call)
        y = layer(x, logits)
        torch.cuda.synchronize()
        check_errors()
        rows = torch.arange(0, T, T // 16, device="cuda")
        ref = reference_moe(x, logits, k, layer.w_gate, layer.w_up, layer.w2, rows)
        got = y[rows].float()
        rel = ((got - ref).norm() / ref.norm()).item()
        assert rel < 2e-2, (call, rel)


@pytest.mark.parametrize("dispatch_ctas,combine_ctas", [(8, 0), (0, 8), (8, 8)])
def test_moe_forward_confined_options(dispatch_ctas, combine_ctas):
    """The A/B options that confine NVLink stores to a few CTAs (dynamic tiles in both grouped
    GEMMs, combine rows staged locally and queued) give the same result as the reference."""
    from opengda_b200.models.moe import MoELayer, make_inputs, reference_moe
    from opengda_b200.ops.gemm import check_errors
    T, H, E, k, I = 512, 1024, 32, 8, 512
    layer = MoELayer(T, H, E, k, I, rt=None, weight_std=0.05)
    layer.dispatch_ctas = dispatch_ctas
    layer.combine_ctas = combine_ctas
    for call in range(3):  # both parities of the tile counters, then the first again
        x, logits = make_inputs(T, H, E, 0, seed=20 + call)
        y = layer(x, logits)
        torch.cuda.synchronize()
        check_errors()
        rows = torch.arange(0, T, T // 16, device="cuda")
        ref = reference_moe(x, logits, k, layer.w_gate, layer.w_up, layer.w2, rows)
        rel = ((y[rows].float() - ref).norm() / ref.norm()).item()
        assert rel < 2e-2, (call, rel)
