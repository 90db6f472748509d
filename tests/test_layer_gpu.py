"""TritonMoEMLP on the GPU: forward + backward of the whole layer.

* Golden: the layer body driven with the reference run's own routing choice
  (selected experts + weights from the fp32 reference golden vectors) must
  match the reference's fp32 outputs and gradients within the bf16
  bound |a - b| <= 1e-2 * scale + 2e-2 * |b| (bf16 storage vs fp32).
* Oracle: at the benchmark bf16 shapes (README uniform / variable, the 768-hidden
  variable config) the module's output and gradients match the CPU oracle run
  on the module's own routing with the reference's bf16 rounding points.
* Properties: determinism, dtypes/shapes, aux losses, state_dict layout.
"""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests.goldens import load
from tests.test_api_gpu import assert_close_scaled

pytestmark = pytest.mark.gpu

LAYER = load("layer")


def widths_of(sizes):
    return [int(w) for c, w in sizes for _ in range(int(c))]


def make_layer(n_embd, expert_sizes, top_k, block_size=64, seed=0, dtype=torch.bfloat16, device="cuda"):
    from moe_b200 import TritonMoEConfig, TritonMoEMLP

    torch.manual_seed(seed)
    m = TritonMoEMLP(TritonMoEConfig(n_embd=n_embd, expert_sizes=expert_sizes,
                                     num_active_experts=top_k, block_size=block_size))
    with torch.no_grad():
        m.router.weight.normal_(0, 0.02)
        m.w1.normal_(0, 0.02)
        m.w2.normal_(0, 0.02)
    return m.to(device=device, dtype=dtype)


@pytest.mark.parametrize("case", sorted(LAYER))
def test_layer_body_matches_reference_golden(case, device):
    from moe_b200.moe import _MoEMLPFunction

    d = LAYER[case]
    H = int(d["n_embd"])
    sizes = [tuple(int(v) for v in s) for s in d["expert_sizes"]]
    m = make_layer(H, sizes, int(d["top_k"]), int(d["block_size"]), device=device)
    bf = torch.bfloat16
    with torch.no_grad():
        m.w1.copy_(torch.from_numpy(d["w1"]).to(bf))
        m.w2.copy_(torch.from_numpy(d["w2"]).to(bf))
    x = torch.from_numpy(d["x"].reshape(-1, H)).to(device, bf).requires_grad_()
    sel = torch.from_numpy(d["selected"]).to(device)
    w = torch.from_numpy(d["weights"]).to(device, bf)
    out, tpe = _MoEMLPFunction.apply(x, m.w1, m.w2, w, sel, m._plan())
    out.float().sum().backward()
    assert_close_scaled(out.float().cpu(), d["out"].reshape(-1, H), "out")
    assert_close_scaled(x.grad.float().cpu(), d["dx"].reshape(-1, H), "dx")
    assert_close_scaled(m.w1.grad.float().cpu(), d["dw1"], "dw1")
    assert_close_scaled(m.w2.grad.float().cpu(), d["dw2"], "dw2")
    np.testing.assert_array_equal(tpe.cpu().numpy(), np.bincount(d["selected"], minlength=len(tpe)))


SHAPES = [
    # name, n_embd, expert_sizes, top_k, batch, seq, block
    ("readme_uniform", 256, [(8, 512)], 2, 8, 512, 64),
    ("readme_variable", 256, [(4, 512), (4, 256)], 2, 8, 512, 64),
    ("c3_768_variable", 768, [(4, 512), (8, 256), (4, 128)], 2, 8, 1024, 64),
    ("block128_k4", 128, [(4, 256), (4, 128)], 4, 3, 100, 128),
    ("block16_k1", 64, [(3, 48)], 1, 1, 37, 16),
]


@pytest.mark.parametrize("name,H,sizes,k,B,S,bs", SHAPES, ids=[s[0] for s in SHAPES])
def test_layer_matches_oracle(name, H, sizes, k, B, S, bs, device):
    m = make_layer(H, sizes, k, bs, seed=1, device=device)
    g = torch.Generator(device="cpu").manual_seed(2)
    x = torch.randn(B, S, H, generator=g).to(device, torch.bfloat16).requires_grad_()
    gout = torch.randn(B, S, H, generator=g).to(device, torch.bfloat16)
    out, aux, f_i = m(x)
    out.backward(gout)
    inter = m.forward_with_intermediates(x.detach())
    sel = inter["selected_experts_flat"].cpu().numpy()
    wts = inter["top_k_weights_flat"].detach().float().cpu().numpy()
    ref = orc.moe_mlp(x.detach().float().cpu().numpy().reshape(-1, H),
                      m.w1.detach().float().cpu().numpy(), m.w2.detach().float().cpu().numpy(),
                      sel, wts, widths_of(sizes), k, bs,
                      grad_out=gout.float().cpu().numpy().reshape(-1, H), dtype="bf16")
    assert_close_scaled(out.detach().float().cpu().reshape(-1, H), ref["out"], f"{name}.out")
    assert_close_scaled(x.grad.float().cpu().reshape(-1, H), ref["dx"], f"{name}.dx")
    assert_close_scaled(m.w1.grad.float().cpu(), ref["dw1"], f"{name}.dw1")
    assert_close_scaled(m.w2.grad.float().cpu(), ref["dw2"], f"{name}.dw2")
    # reference-layout intermediates agree with the fused path
    assert_close_scaled(inter["output"].float().cpu().reshape(-1, H), ref["out"], f"{name}.inter.out")
    np.testing.assert_array_equal(inter["tokens_per_expert"].cpu().numpy(),
                                  ref["routing"]["tokens_per_expert"])
    assert out.dtype == torch.bfloat16 and out.shape == x.shape
    assert f_i.shape == (m.num_experts,) and abs(float(f_i.float().sum()) - 1.0) < 1e-2
    for v in aux.values():
        assert torch.isfinite(v).all()


def test_layer_is_deterministic(device):
    m = make_layer(256, [(4, 512), (4, 256)], 2, device=device)
    x = torch.randn(4, 256, 256, device=device, dtype=torch.bfloat16)
    outs = []
    for _ in range(2):
        m.zero_grad(set_to_none=True)
        xi = x.clone().requires_grad_()
        o, _, _ = m(xi)
        o.float().sum().backward()
        outs.append((o.detach(), xi.grad, m.w1.grad.clone(), m.w2.grad.clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_aux_losses_match_reference_formulas(device):
    """Fused router head + aux-loss kernels against the reference's fp32 golden
    values (config c1v: variable widths, two size groups)."""
    d = LAYER["c1v"]
    H = int(d["n_embd"])
    sizes = [tuple(int(v) for v in s) for s in d["expert_sizes"]]
    m = make_layer(H, sizes, int(d["top_k"]), int(d["block_size"]), device=device, dtype=torch.float32)
    with torch.no_grad():
        m.router.weight.copy_(torch.from_numpy(d["router_w"]))
    x = torch.from_numpy(d["x"]).to(device)
    logits, probs, w, sel, lse, head_losses = m._route_weights(x.reshape(-1, H))
    np.testing.assert_array_equal(sel.reshape(-1).cpu().numpy(), d["selected"])
    np.testing.assert_allclose(w.reshape(-1).cpu().numpy(), d["weights"], rtol=1e-6, atol=1e-7)
    aux, f_i = m._aux_losses(logits, lse, head_losses, probs)
    np.testing.assert_allclose(f_i.cpu().numpy(), d["f_i"], rtol=1e-6)
    np.testing.assert_allclose(aux["router_z_loss"].item(), d["z_loss"], rtol=1e-5)
    np.testing.assert_allclose(aux["load_balance_loss"].item(), d["lb_loss"], rtol=1e-5)
    np.testing.assert_allclose(aux["compute_loss"].item(), d["compute_loss"], rtol=1e-5)


@pytest.mark.parametrize("sizes,dtype", [([(4, 128)], torch.bfloat16), ([(2, 128), (3, 64), (1, 256)], torch.bfloat16),
                                         ([(1, 128), (1, 64)], torch.float32), ([(4, 512), (8, 256), (4, 128)], torch.bfloat16)])
def test_aux_losses_forward_and_gradients_match_torch(sizes, dtype, device):
    """The fused aux losses and their gradients w.r.t. the router weight equal
    the reference's torch expressions evaluated by autograd."""
    H, k = 64, 2
    E = sum(c for c, _ in sizes)
    m = make_layer(H, sizes, min(k, E), 64, device=device, dtype=dtype)
    x = torch.randn(300, H, device=device, dtype=dtype)
    logits, probs, w, sel, lse, head_losses = m._route_weights(x)
    from moe_b200.kernels import fused_route

    _, _, tpe, _, _ = fused_route(sel.reshape(-1), E)
    aux, f_i = m._aux_losses(logits, lse, head_losses, probs)
    (aux["router_z_loss"].float() + aux["load_balance_loss"] + aux["compute_loss"]).backward()
    g_fused = m.router.weight.grad.float().clone()
    m.router.weight.grad = None
    lg = m.router(x)
    pr = torch.sigmoid(lg.float())
    from oracle import aux_reference

    ref, f_ref = aux_reference.aux_losses(sizes, lg, pr, tpe, dtype)
    (ref["router_z_loss"].float() + ref["load_balance_loss"] + ref["compute_loss"]).backward()
    g_ref = m.router.weight.grad.float()
    assert torch.equal(f_i, f_ref)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    for key in aux:
        torch.testing.assert_close(aux[key].float(), ref[key].float(), rtol=tol, atol=1e-6)
    torch.testing.assert_close(g_fused, g_ref, rtol=5e-2, atol=1e-2 * g_ref.abs().max().item())


@pytest.mark.parametrize("T,E,k", [(300, 6, 2), (8192, 16, 2), (20000, 64, 8), (5, 3, 1)])
def test_fused_head_losses_match_separate_launches(T, E, k, device):
    """moe_router_head_losses (head + losses in one launch, expert counts taken
    from the head's own selections) equals moe_router_head + moe_aux_losses with
    the routing's tokens_per_expert, and leaves its ticket at zero."""
    from moe_b200.kernels import _ops, fused_route

    g = torch.Generator(device="cpu").manual_seed(T + E)
    logits = torch.randn(T, E, generator=g).to(device, torch.bfloat16)
    wn = torch.rand(E, generator=g).to(device)
    coef = torch.rand(E, generator=g).to(device)
    ticket = torch.zeros(1, dtype=torch.int32, device=device)
    for _ in range(3):  # the ticket is reused across calls
        probs, w, sel, lse, ws, (losses, f_i, p_i, z) = _ops.router_head(
            logits, k, True, torch.bfloat16, wn, coef, ticket)
        probs2, w2, sel2, lse2, ws2 = _ops.router_head(logits, k, True, torch.bfloat16, wn)
        _, _, tpe, _, _ = fused_route(sel2.reshape(-1), E)
        losses2, f2, p2, z2 = _ops.aux_losses(ws2, T, tpe, coef, torch.bfloat16, torch.bfloat16)
        # the head's own selection counts stand in for tokens_per_expert
        losses3, f3, p3, z3 = _ops.aux_losses(ws2, T, None, coef, torch.bfloat16, torch.bfloat16)
        torch.cuda.synchronize()
        assert torch.equal(losses3, losses2) and torch.equal(f3, f2) and torch.equal(z3, z2)
        assert int(ticket.item()) == 0
        assert torch.equal(sel, sel2) and torch.equal(w, w2) and torch.equal(probs, probs2)
        assert torch.equal(f_i, f2)
        torch.testing.assert_close(p_i, p2, rtol=1e-6, atol=0)
        torch.testing.assert_close(losses, losses2, rtol=1e-6, atol=0)
        assert torch.equal(z, z2)


def test_state_dict_layout_matches_reference(device):
    m = make_layer(64, [(2, 128), (2, 64)], 2, device=device)
    sd = m.state_dict()
    assert sorted(sd) == ["router.weight", "w1", "w2"]
    assert sd["w1"].shape == (64, 384) and sd["w2"].shape == (384, 64)
    assert sd["router.weight"].shape == (4, 64)
