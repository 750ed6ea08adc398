"""CPU checks of the MoE layer's host helpers: the gate/up interleave of W1 and the fp32
reference layer used as the oracle of the GPU tests."""
import torch

from opengda_b200.models.moe import interleave_w1, reference_moe


def test_interleave_w1_blocks_of_128():
    E, I, H = 2, 256, 8
    g = torch.arange(E * I * H, dtype=torch.float32).view(E, I, H)
    u = -g
    w = interleave_w1(g, u)
    assert w.shape == (E, 2 * I, H)
    for e in range(E):
        for b in range(I // 128):
            assert torch.equal(w[e, 256 * b:256 * b + 128], g[e, 128 * b:128 * b + 128])
            assert torch.equal(w[e, 256 * b + 128:256 * b + 256], u[e, 128 * b:128 * b + 128])


def test_reference_matches_a_batched_restatement():
    torch.manual_seed(0)
    T, H, E, k, I = 6, 16, 5, 2, 8
    x = torch.randn(T, H)
    logits = torch.randn(T, E)
    wg, wu, w2 = torch.randn(E, I, H), torch.randn(E, I, H), torch.randn(E, H, I)
    got = reference_moe(x, logits, k, wg, wu, w2)
    prob = torch.softmax(logits, -1)
    w, idx = torch.topk(prob, k, -1)
    gate = torch.einsum("tkih,th->tki", wg[idx], x)
    up = torch.einsum("tkih,th->tki", wu[idx], x)
    y = torch.einsum("tkhi,tki->tkh", w2[idx], torch.nn.functional.silu(gate) * up)
    ref = (w.unsqueeze(-1) * y).sum(1)
    assert torch.allclose(got, ref, rtol=1e-4, atol=1e-4)
    rows = torch.tensor([1, 4])
    assert torch.allclose(reference_moe(x, logits, k, wg, wu, w2, rows), ref[rows], rtol=1e-4, atol=1e-4)
