"""Fused top-k + renormalisation of the router probabilities against the
reference's torch ops (triton_moe/moe.py:168-182): same experts in the same
order (bit-exact), same weights (bit-exact when the top-k sum is exact, within
one bf16 ulp otherwise), equal probabilities resolved to the lower index."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def torch_reference(probs, k, norm, dtype):
    w, sel = torch.topk(probs, k, dim=-1)
    if norm:
        w = w / (w.sum(dim=-1, keepdim=True) + 1e-20)
    return w.to(dtype), sel


@pytest.mark.parametrize("T,E,k", [(1, 4, 2), (8192, 16, 2), (1000, 64, 8), (333, 128, 8),
                                   (77, 256, 8), (50, 33, 32), (5, 7, 7)])
@pytest.mark.parametrize("norm", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_router_topk_matches_torch(T, E, k, norm, dtype, device):
    from moe_b200.kernels import _ops

    g = torch.Generator(device="cpu").manual_seed(T * 131 + E)
    # a random permutation per row: every probability distinct
    probs = torch.sigmoid(torch.argsort(torch.rand(T, E, generator=g), dim=-1).float() / E - 0.5)
    probs = probs.to(device)
    w, sel = _ops.router_topk(probs, k, norm, dtype)
    w_ref, sel_ref = torch_reference(probs, k, norm, dtype)
    assert torch.equal(sel.long(), sel_ref)
    if k <= 2 or not norm:
        assert torch.equal(w, w_ref)
    else:
        torch.testing.assert_close(w.float(), w_ref.float(), rtol=8e-3, atol=0)


def test_router_topk_ties_go_to_lower_index(device):
    from moe_b200.kernels import _ops

    probs = torch.tensor([[0.5, 0.7, 0.7, 0.1, 0.7], [0.2, 0.2, 0.2, 0.2, 0.2]], device=device)
    w, sel = _ops.router_topk(probs, 2, True, torch.float32)
    assert sel.tolist() == [[1, 2], [0, 1]]
    assert torch.allclose(w, torch.full_like(w, 0.5))
