"""The layer at the large benchmark shapes (c4: 2048 hidden, 64 experts,
top-8, Zipf-skewed routing; and a 4096-hidden, 128-expert variable layer at a
reduced token count) against a plain PyTorch fp32 reference of the same
routing, computed expert by expert on the GPU.  Tolerance (bf16 storage):
|a-b| <= 1e-2 * max|b| + 2e-2 |b|."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(a, b, what):
    a, b = a.float(), b.float()
    scale = b.abs().max().clamp_min(1e-30)
    bad = (a - b).abs() > 1e-2 * scale + 2e-2 * b.abs()
    assert not bad.any(), f"{what}: {int(bad.sum())}/{bad.numel()} mismatches, max err {(a - b).abs().max():.3e} scale {scale:.3e}"


def _reference(layer, x_flat, gout, sel, w):
    """fp32 dense restatement: out = sum_j w_j relu(x W1_e)^2 W2_e (weights detached)."""
    H = x_flat.shape[1]
    x = x_flat.float().detach().requires_grad_()
    w1 = layer.w1.detach().float().requires_grad_()
    w2 = layer.w2.detach().float().requires_grad_()
    out = torch.zeros_like(x)
    offs = [0]
    for wd in layer.expert_widths:
        offs.append(offs[-1] + wd)
    for e in range(layer.num_experts):
        tok, slot = (sel == e).nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        h = torch.relu(x[tok] @ w1[:, offs[e]:offs[e + 1]]) ** 2
        out = out.index_add(0, tok, (h @ w2[offs[e]:offs[e + 1]]) * w[tok, slot, None].float())
    out.backward(gout.float())
    return out.detach(), x.grad, w1.grad, w2.grad


@pytest.mark.parametrize("H,sizes,k,T,zipf", [
    (2048, [(64, 1024)], 8, 16384, True),
    (4096, [(32, 2048), (64, 1024), (32, 512)], 8, 4096, True),
])
def test_large_layer_matches_fp32_reference(H, sizes, k, T, zipf, device):
    from moe_b200 import TritonMoEConfig, TritonMoEMLP

    torch.manual_seed(0)
    m = TritonMoEMLP(TritonMoEConfig(n_embd=H, expert_sizes=sizes, num_active_experts=k,
                                     block_size=64))
    with torch.no_grad():
        for p in (m.router.weight, m.w1, m.w2):
            p.normal_(0, 0.02)
    E = m.num_experts
    if zipf:  # skewed routing: a Zipf(1.1) prior as a router bias
        r = torch.nn.Linear(H, E, bias=True)
        ranks = torch.randperm(E).float() + 1
        lp = -1.1 * torch.log(ranks)
        with torch.no_grad():
            r.weight.copy_(m.router.weight)
            r.bias.copy_(lp - lp.mean())
        m.router = r
    m = m.to(device, torch.bfloat16)
    g = torch.Generator(device="cpu").manual_seed(1)
    x = torch.randn(1, T, H, generator=g).to(device, torch.bfloat16).requires_grad_()
    gout = torch.randn(1, T, H, generator=g).to(device, torch.bfloat16)
    out, aux, f_i = m(x)
    out.backward(gout)
    torch.cuda.synchronize()
    _, _, w, sel, _, _ = m._route_weights(x.detach().reshape(T, H))
    ro, rdx, rw1, rw2 = _reference(m, x.detach().reshape(T, H), gout.reshape(T, H), sel.long(), w)
    _close(out.reshape(T, H), ro, "out")
    _close(x.grad.reshape(T, H), rdx, "dx")
    _close(m.w1.grad, rw1, "dw1")
    _close(m.w2.grad, rw2, "dw2")
    tpe = torch.bincount(sel.reshape(-1).long(), minlength=E)
    assert tpe.max() > 2 * tpe.float().mean() or not zipf  # routing really is skewed
