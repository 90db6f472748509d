"""Reference-facing API on the GPU against the reference's golden vectors and
the CPU oracle.

* permutation ops (gather / weighted gather / scatter / gather map) in fp32:
  the golden vectors must be reproduced exactly (copies) or to fp32 rounding;
* the same ops in bf16: bit-exact against the oracle's bf16 restatement;
* the grouped GEMM API (up / down / both backwards, with and without the
  fused-gather map) in bf16 on the golden inputs: within the bf16 bound
  |a - b| <= 1e-2 * scale + 2e-2 * |b| of the oracle run in fp32 on the same
  bf16-rounded inputs, where scale = max |b| of the tensor (the golden values
  are O(1e-1), so a bare 1e-2 absolute bound would be vacuous).
"""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests.goldens import load

pytestmark = pytest.mark.gpu

RTOL, ATOL_REL = 2e-2, 1e-2


def assert_close_scaled(a, b, what):
    if isinstance(a, torch.Tensor):
        a = a.detach().float().cpu().numpy()
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    assert a.shape == b.shape, f"{what}: shape {a.shape} vs {b.shape}"
    scale = max(np.abs(b).max(initial=0.0), 1e-30)
    bad = np.abs(a - b) > ATOL_REL * scale + RTOL * np.abs(b)
    assert not bad.any(), (
        f"{what}: {bad.sum()} / {bad.size} outside tolerance; max err "
        f"{np.abs(a - b).max():.3e}, scale {scale:.3e}"
    )


def T(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t.to(dtype) if dtype is not None else t


def test_permutation_fp32_matches_golden(device):
    from moe_b200.kernels import padded_gather, padded_scatter, precompute_gather_map
    from moe_b200.kernels.gather import _weighted_padded_gather

    d = load("permute")
    k = int(d["top_k"])
    meta = [T(d[n], device) for n in ("indices", "bin_ids", "bins", "padded_bins")]
    x, w, y = T(d["x"], device), T(d["w"], device), T(d["y"], device)
    np.testing.assert_array_equal(padded_gather(x, *meta, k).cpu().numpy(), d["gathered"])
    np.testing.assert_array_equal(
        _weighted_padded_gather(x, meta[0], meta[1], w, meta[2], meta[3], k).cpu().numpy(),
        d["weighted_gathered"])
    np.testing.assert_allclose(
        padded_scatter(y, meta[0], meta[1], w, meta[2], meta[3], k).cpu().numpy(),
        d["scattered"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(precompute_gather_map(*meta, k).cpu().numpy(), d["gather_map"])


@pytest.mark.parametrize("H", [40, 256])  # scalar and 128-bit paths
def test_permutation_bf16_bit_exact_vs_oracle(H, device):
    from moe_b200.kernels import fused_route, padded_gather, padded_scatter
    from moe_b200.kernels.gather import _weighted_padded_gather

    rng = np.random.default_rng(3)
    Tn, k, E, bs = 333, 4, 12, 64
    sel = rng.integers(0, E, Tn * k)
    x = orc.round_bf16(rng.standard_normal((Tn, H)).astype(np.float32))
    w = orc.round_bf16(rng.random(Tn * k).astype(np.float32))
    r = orc.fused_route(sel, E, bs)
    args = (r["indices"], r["bin_ids"], r["bins"], r["padded_bins"])
    bid, ind, tpe, bins, pb = fused_route(T(sel, device), E, bs)
    g = padded_gather(T(x, device, torch.bfloat16), ind, bid, bins, pb, k)
    np.testing.assert_array_equal(g.float().cpu().numpy(), orc.padded_gather(x, *args, k, dtype="bf16"))
    gw = _weighted_padded_gather(T(x, device, torch.bfloat16), ind, bid, T(w, device, torch.bfloat16),
                                 bins, pb, k)
    np.testing.assert_array_equal(gw.float().cpu().numpy(),
                                  orc.padded_gather(x, *args, k, weights=w, dtype="bf16"))
    y = orc.round_bf16(rng.standard_normal((int(r["padded_bins"][-1]), H)).astype(np.float32))
    s = padded_scatter(T(y, device, torch.bfloat16), ind, bid, T(w, device, torch.bfloat16), bins, pb, k)
    np.testing.assert_array_equal(
        s.float().cpu().numpy(),
        orc.padded_scatter(y, r["indices"], r["bin_ids"], w, r["bins"], r["padded_bins"], k, dtype="bf16"))


GEMM = load("gemm")


@pytest.mark.parametrize("case", sorted(GEMM))
def test_grouped_gemm_api_bf16_vs_golden_inputs(case, device):
    from moe_b200 import kernels as K

    d = GEMM[case]
    bf = torch.bfloat16
    q = {n: orc.round_bf16(d[n]) for n in ("x", "w1", "w2", "gy", "x_flat")}
    to, wo = d["tok_off"], d["w_off"]
    widths = d["widths"].astype(np.int32)
    maxw = int(widths.max())
    H = int(d["H"])
    tt = dict(tok=T(to, device), wo=T(wo, device), widths=T(widths, device),
              tpe=T(d["counts"].astype(np.int32), device))
    x, w1, w2 = T(q["x"], device, bf), T(q["w1"], device, bf), T(q["w2"], device, bf)
    args = (tt["tok"], tt["wo"], tt["widths"], tt["tpe"])

    out, pre = K.grouped_gemm_up(x, w1, *args, maxw, activation="relu_squared", save_pre_act=True)
    o_out, o_pre = orc.grouped_gemm_up(q["x"], q["w1"], to, wo, maxw, "relu_squared")
    assert_close_scaled(out.float().cpu(), o_out, "up.out")
    assert_close_scaled(pre.float().cpu(), o_pre, "up.pre")
    assert_close_scaled(out.float().cpu(), d["out"], "up.out vs fp32 golden")

    hq = orc.round_bf16(out.float().cpu().numpy())
    y = K.grouped_gemm_down(out, w2, *args, H)
    assert_close_scaled(y.float().cpu(), orc.grouped_gemm_down(hq, q["w2"], to, wo), "down")

    gy = T(q["gy"], device, bf)
    gi, gw2 = K.grouped_gemm_down_backward(gy, out, w2, *args, H, maxw)
    o_gi, o_gw2 = orc.grouped_gemm_down_backward(q["gy"], hq, q["w2"], to, wo, maxw)
    assert_close_scaled(gi.float().cpu(), o_gi, "down.dinter")
    assert_close_scaled(gw2.float().cpu(), o_gw2, "down.dw")

    giq = orc.round_bf16(gi.float().cpu().numpy())
    preq = orc.round_bf16(pre.float().cpu().numpy())
    gx, gw1 = K.grouped_gemm_up_backward(gi, x, w1, pre, *args, H, "relu_squared")
    o_gx, o_gw1 = orc.grouped_gemm_up_backward(giq, q["x"], q["w1"], preq, to, wo, dtype="bf16")
    assert_close_scaled(gx.float().cpu(), o_gx, "up.dx")
    assert_close_scaled(gw1.float().cpu(), o_gw1, "up.dw")

    # fused-gather variants (x_flat + gather_map)
    xf = T(q["x_flat"], device, bf)
    gm = T(d["gmap"], device)
    out_gm = K.grouped_gemm_up(xf, w1, *args, maxw, activation="relu_squared", gather_map=gm)
    o_gm, _ = orc.grouped_gemm_up(q["x_flat"], q["w1"], to, wo, maxw, "relu_squared",
                                  gather_map=d["gmap"])
    assert_close_scaled(out_gm.float().cpu(), o_gm, "up.gather_map")
    gx2, gw1_2 = K.grouped_gemm_up_backward(gi, xf, w1, pre, *args, H, "relu_squared", gather_map=gm)
    o_gx2, o_gw1_2 = orc.grouped_gemm_up_backward(giq, q["x_flat"], q["w1"], preq, to, wo,
                                                  gather_map=d["gmap"], dtype="bf16")
    assert_close_scaled(gx2.float().cpu(), o_gx2, "up.dx.gather_map")
    assert_close_scaled(gw1_2.float().cpu(), o_gw1_2, "up.dw.gather_map")


def test_autograd_functions_match_direct_calls(device):
    """GroupedGemmUp/Down autograd == the direct forward/backward functions
    (the reference's self-consistency test, test_grouped_gemm_backward.py:132-249)."""
    from moe_b200 import kernels as K

    g = torch.Generator(device="cpu").manual_seed(0)
    H, E, n = 64, 2, 128
    widths = torch.tensor([128, 128], dtype=torch.int32, device=device)
    tok = torch.tensor([0, n, 2 * n], dtype=torch.int32, device=device)
    wo = torch.tensor([0, 128, 256], dtype=torch.int32, device=device)
    tpe = torch.tensor([n, n], dtype=torch.int32, device=device)
    x = torch.randn(2 * n, H, generator=g).bfloat16().to(device).requires_grad_()
    w1 = (torch.randn(H, 256, generator=g) * 0.1).bfloat16().to(device).requires_grad_()
    w2 = (torch.randn(256, H, generator=g) * 0.1).bfloat16().to(device).requires_grad_()
    h = K.grouped_gemm_up_autograd(x, w1, tok, wo, widths, tpe, 128, H)
    y = K.grouped_gemm_down_autograd(h, w2, tok, wo, widths, tpe, H, 128)
    y.float().sum().backward()
    h_d = K.grouped_gemm_up(x.detach(), w1.detach(), tok, wo, widths, tpe, 128)
    assert torch.equal(h.detach(), h_d)
    assert torch.equal(y.detach(), K.grouped_gemm_down(h_d, w2.detach(), tok, wo, widths, tpe, H))
    for p in (x, w1, w2):
        assert p.grad is not None and torch.isfinite(p.grad.float()).all() and p.grad.abs().sum() > 0
