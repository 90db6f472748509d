"""fp32 operands: the grouped GEMMs run on the tf32 tensor-core MMA
(tcgen05 kind::tf32, fp32 accumulation), the reference's own default for fp32
dots.  Checked against

* a plain PyTorch fp32 reference, expert by expert, for all six GEMMs and both
  fused epilogues, including k tails that are not a multiple of the 32-wide
  fp32 k-block; tolerance |a-b| <= 1e-2 * scale + 1e-2 |b| (tf32 keeps 10
  mantissa bits, so each product carries ~5e-4 relative error);
* the reference's fp32 golden vectors for the whole layer (forward with its
  own routing, and all gradients), within |a - b| <= 1e-2 * scale + 2e-2 * |b|.
"""

import math

import numpy as np
import pytest
import torch

from tests.goldens import load
from tests.test_api_gpu import assert_close_scaled
from tests.test_grouped_gemm_gpu import CASES, make_problem

pytestmark = pytest.mark.gpu

F32 = torch.float32


def close(a, b, what):
    a, b = a.float(), b.float()
    scale = max(b.abs().max().item(), 1e-30)
    bad = (a - b).abs() > 1e-2 * scale + 1e-2 * b.abs()
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{bad.numel()} outside tolerance, max err "
                           f"{(a - b).abs().max().item():.3e}, scale {scale:.3e}")


FP32_CASES = CASES + [([48, 16, 112], [33, 17, 70], 80, 16)]  # k tails of 16 in both GEMMs


@pytest.mark.parametrize("case", FP32_CASES, ids=[f"c{i}" for i in range(len(FP32_CASES))])
@pytest.mark.parametrize("tile_n", [128, 256, 128 | 0x200, 256 | 0x200])
def test_fp32_forward(case, tile_n, device):
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, dtype=F32, device=device, seed=11)
    args = (m["tok_off"], m["w_off"], m["tpe"], m["E"])
    out = torch.zeros(m["rows"], m["maxw"], dtype=F32, device=device)
    pre = torch.zeros_like(out)
    _ops.gemm_up(t["x"], t["w1"], *args, "relu_squared", out, pre, tile_n=tile_n)
    y = torch.zeros(m["rows"], H, dtype=F32, device=device)
    _ops.gemm_down(t["ga"], t["w2"], *args, y, tile_n=tile_n)
    torch.cuda.synchronize()
    _ops.check_device_status(device)
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        if r1 == r0:
            continue
        z = t["x"][r0:r1] @ t["w1"][:, c0:c1]
        close(pre[r0:r1, : c1 - c0], torch.relu(z), f"pre e{e}")
        close(out[r0:r1, : c1 - c0], torch.relu(z) ** 2, f"out e{e}")
        assert (out[r0:r1, c1 - c0:] == 0).all()
        close(y[r0:r1], t["ga"][r0:r1, : c1 - c0] @ t["w2"][c0:c1], f"y e{e}")


@pytest.mark.parametrize("case", FP32_CASES, ids=[f"c{i}" for i in range(len(FP32_CASES))])
@pytest.mark.parametrize("pair", [0, 0x200])
def test_fp32_backward(case, pair, device):
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, dtype=F32, device=device, seed=12)
    args = (m["tok_off"], m["w_off"], m["tpe"], m["E"])
    dact = torch.zeros(m["rows"], m["maxw"], dtype=F32, device=device)
    gw2 = torch.full((m["TW"], H), 7.0, dtype=F32, device=device)
    _ops.gemm_down_backward(t["gy"], t["ga"], t["w2"], *args, dact, gw2, pre_act=t["pre"],
                            tile_n_width=128 | pair, tile_n_hidden=256 | pair)
    gx = torch.zeros(m["rows"], H, dtype=F32, device=device)
    gw1 = torch.full((H, m["TW"]), 7.0, dtype=F32, device=device)
    _ops.gemm_up_backward(t["ga"], t["x"], t["w1"], *args, gx, gw1, tile_n_width=128 | pair,
                          tile_n_hidden=256 | pair)
    torch.cuda.synchronize()
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        ga = t["ga"][r0:r1, : c1 - c0]
        close(gw2[c0:c1], ga.T @ t["gy"][r0:r1], f"gw2 e{e}")
        close(gw1[:, c0:c1], t["x"][r0:r1].T @ ga, f"gw1 e{e}")
        if r1 == r0:
            continue
        g = t["gy"][r0:r1] @ t["w2"][c0:c1].T
        p = t["pre"][r0:r1, : c1 - c0]
        close(dact[r0:r1, : c1 - c0], torch.where(p > 0, g * 2.0 * p, torch.zeros_like(p)),
              f"dact e{e}")
        close(gx[r0:r1], ga @ t["w1"][:, c0:c1].T, f"gx e{e}")


LAYER = load("layer")


@pytest.mark.parametrize("case", sorted(LAYER))
def test_fp32_layer_matches_reference_golden(case, device):
    """The whole fp32 layer (router, routing, MLP, backward) reproduces the
    reference's fp32 run: same expert choice, outputs and gradients in bound."""
    from moe_b200 import TritonMoEConfig, TritonMoEMLP

    d = LAYER[case]
    H = int(d["n_embd"])
    sizes = [tuple(int(v) for v in s) for s in d["expert_sizes"]]
    norm = bool(int(d["norm_topk_prob"])) if "norm_topk_prob" in d else True
    m = TritonMoEMLP(TritonMoEConfig(n_embd=H, expert_sizes=sizes,
                                     num_active_experts=int(d["top_k"]),
                                     norm_topk_prob=norm,
                                     block_size=int(d["block_size"]))).to(device)
    with torch.no_grad():
        m.router.weight.copy_(torch.from_numpy(d["router_w"]))
        m.w1.copy_(torch.from_numpy(d["w1"]))
        m.w2.copy_(torch.from_numpy(d["w2"]))
    x = torch.from_numpy(d["x"]).to(device).requires_grad_()
    inter = m.forward_with_intermediates(x.detach())
    np.testing.assert_array_equal(inter["selected_experts_flat"].cpu().numpy(),
                                  d["selected"].reshape(-1))
    out, aux, f_i = m(x)
    assert out.dtype == F32
    assert_close_scaled(out.detach().cpu().reshape(-1, H), d["out"].reshape(-1, H), "out")
    out.sum().backward()
    # the golden gradients are those of out.sum() alone
    assert_close_scaled(x.grad.cpu().reshape(-1, H), d["dx"].reshape(-1, H), "dx")
    assert_close_scaled(m.w1.grad.cpu(), d["dw1"], "dw1")
    assert_close_scaled(m.w2.grad.cpu(), d["dw2"], "dw2")
    np.testing.assert_allclose(float(aux["router_z_loss"].detach()), float(d["z_loss"]), rtol=1e-4)
