"""Pins the CPU oracle to the reference: every golden vector produced by the
reference's own Triton kernels (TRITON_INTERPRET=1, fp32) must be reproduced.
Integer outputs bit-exact; fp32 outputs to 1e-5 relative of the tensor scale
(the two differ only in fp32 summation order)."""

import numpy as np
import pytest

from oracle import moe_oracle as orc
from tests.goldens import load


def close(a, b, what, rtol=1e-5):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    assert a.shape == b.shape, f"{what}: shape {a.shape} vs {b.shape}"
    scale = max(np.abs(b).max(initial=0.0), 1e-30)
    err = np.abs(a - b).max(initial=0.0)
    assert err <= rtol * scale, f"{what}: max err {err:.3e} vs scale {scale:.3e}"


ROUTE = load("route")


@pytest.mark.parametrize("case", sorted(ROUTE))
def test_route_matches_reference(case):
    d = ROUTE[case]
    r = orc.fused_route(d["sel"], int(d["E"]), int(d["bs"]), str(d["rounding"]))
    for k in ("bin_ids", "indices", "tokens_per_expert", "bins", "padded_bins"):
        np.testing.assert_array_equal(r[k], d[k], err_msg=f"{case}:{k}")


def test_permutation_matches_reference():
    d = load("permute")
    k = int(d["top_k"])
    args = (d["indices"], d["bin_ids"], d["bins"], d["padded_bins"])
    close(orc.padded_gather(d["x"], *args, k), d["gathered"], "gather", rtol=0)
    close(orc.padded_gather(d["x"], *args, k, weights=d["w"]), d["weighted_gathered"], "wgather")
    close(orc.padded_scatter(d["y"], d["indices"], d["bin_ids"], d["w"], d["bins"],
                             d["padded_bins"], k), d["scattered"], "scatter")
    np.testing.assert_array_equal(orc.precompute_gather_map(*args, k), d["gather_map"])


GEMM = load("gemm")


@pytest.mark.parametrize("case", sorted(GEMM))
def test_grouped_gemms_match_reference(case):
    d = GEMM[case]
    to, wo, maxw = d["tok_off"], d["w_off"], int(d["widths"].max())
    out, pre = orc.grouped_gemm_up(d["x"], d["w1"], to, wo, maxw, "relu_squared")
    close(out, d["out"], "up.out")
    close(pre, d["pre"], "up.pre")
    out_none, _ = orc.grouped_gemm_up(d["x"], d["w1"], to, wo, maxw, "none")
    close(out_none, d["out_none"], "up.none")
    close(orc.grouped_gemm_down(d["out"], d["w2"], to, wo), d["y"], "down")
    gi, gw2 = orc.grouped_gemm_down_backward(d["gy"], d["out"], d["w2"], to, wo, maxw)
    close(gi, d["gi"], "down.dinter")
    close(gw2, d["gw2"], "down.dw")
    gx, gw1 = orc.grouped_gemm_up_backward(d["gi"], d["x"], d["w1"], d["pre"], to, wo)
    close(gx, d["gx"], "up.dx")
    close(gw1, d["gw1"], "up.dw")
    out_gm, _ = orc.grouped_gemm_up(d["x_flat"], d["w1"], to, wo, maxw, "relu_squared",
                                    gather_map=d["gmap"])
    close(out_gm, d["out_gm"], "up.gather_map")
    gx_gm, gw1_gm = orc.grouped_gemm_up_backward(d["gi"], d["x_flat"], d["w1"], d["pre"], to, wo,
                                                 gather_map=d["gmap"])
    close(gx_gm, d["gx_gm"], "up.dx.gather_map")
    close(gw1_gm, d["gw1_gm"], "up.dw.gather_map")


LAYER = load("layer")


def expert_widths(sizes):
    return [int(w) for c, w in sizes for _ in range(int(c))]


@pytest.mark.parametrize("case", sorted(LAYER))
def test_layer_forward_backward_matches_reference(case):
    d = LAYER[case]
    H = int(d["n_embd"])
    x = d["x"].reshape(-1, H)
    res = orc.moe_mlp(x, d["w1"], d["w2"], d["selected"], d["weights"],
                      expert_widths(d["expert_sizes"]), int(d["top_k"]), int(d["block_size"]),
                      grad_out=np.ones_like(x))
    close(res["out"], d["out"].reshape(-1, H), "out")
    close(res["dx"], d["dx"].reshape(-1, H), "dx")
    close(res["dw1"], d["dw1"], "dw1")
    close(res["dw2"], d["dw2"], "dw2")


SWIGLU = load("swiglu")


@pytest.mark.parametrize("case", sorted(SWIGLU))
def test_swiglu_forward_matches_reference(case):
    """The oracle's swiglu up projection reproduces the reference kernel's
    (run under the Triton interpreter): output silu(gate) * up, pre_act = gate."""
    d = SWIGLU[case]
    maxw = int(d["widths"].max())
    out, pre = orc.grouped_gemm_up(d["x"], d["w1"], d["tok_off"], d["w_off"], maxw, "swiglu")
    scale = max(np.abs(d["out"]).max(), 1e-30)
    np.testing.assert_allclose(out, d["out"], rtol=1e-5, atol=1e-5 * scale)
    np.testing.assert_allclose(pre, d["pre"], rtol=1e-5, atol=1e-5 * max(np.abs(d["pre"]).max(), 1e-30))


def test_swiglu_backward_is_the_gradient():
    """The oracle's swiglu backward equals central differences of silu(g) * u."""
    rng = np.random.default_rng(0)
    g0 = rng.standard_normal((16, 32)).astype(np.float64)
    u0 = rng.standard_normal((16, 32)).astype(np.float64)
    go = rng.standard_normal((16, 32)).astype(np.float64)
    f = lambda g, u: (g / (1 + np.exp(-g)) * u * go).sum()  # noqa: E731
    ga = orc.swiglu_backward(go, g0, u0, [0, 16], [0, 64])
    eps = 1e-4
    for (i, j) in [(0, 0), (3, 7), (15, 31)]:
        dg = np.zeros_like(g0); dg[i, j] = eps
        du = np.zeros_like(u0); du[i, j] = eps
        num_g = (f(g0 + dg, u0) - f(g0 - dg, u0)) / (2 * eps)
        num_u = (f(g0, u0 + du) - f(g0, u0 - du)) / (2 * eps)
        np.testing.assert_allclose(ga[i, j], num_g, rtol=1e-3, atol=1e-4)
        np.testing.assert_allclose(ga[i, 32 + j], num_u, rtol=1e-3, atol=1e-4)


def test_bf16_rounding_is_round_to_nearest_even():
    import torch

    rng = np.random.default_rng(0)
    v = np.concatenate([
        np.array([1.0, 1.00390625, 1.01171875, 1.0 + 2**-9, -2.5e-3, 3.0e38, 0.0, -0.0], np.float32),
        (rng.standard_normal(10000) * 10.0 ** rng.integers(-20, 20, 10000)).astype(np.float32),
    ])
    exp = torch.from_numpy(v).bfloat16().float().numpy()
    np.testing.assert_array_equal(orc.round_bf16(v), exp)


@pytest.mark.parametrize("case", sorted(load("layer")))
def test_aux_loss_checker_matches_reference(case):
    """oracle.aux_reference (the torch checker of the fused aux-loss kernels)
    reproduces the reference layer's z-loss, load-balance loss, compute loss
    and f_i from the golden router weights and tokens."""
    import torch

    from oracle import aux_reference

    d = load("layer")[case]
    sizes = [tuple(int(v) for v in s) for s in d["expert_sizes"]]
    E = sum(c for c, _ in sizes)
    x = torch.from_numpy(d["x"]).reshape(-1, int(d["n_embd"]))
    logits = x @ torch.from_numpy(d["router_w"]).T
    probs = torch.sigmoid(logits)
    tpe = torch.bincount(torch.from_numpy(d["selected"]).reshape(-1).long(), minlength=E)
    aux, f_i = aux_reference.aux_losses(sizes, logits, probs, tpe, torch.float32)
    np.testing.assert_allclose(f_i.numpy(), d["f_i"], rtol=1e-6)
    np.testing.assert_allclose(aux["router_z_loss"].item(), d["z_loss"], rtol=1e-5)
    np.testing.assert_allclose(aux["load_balance_loss"].item(), d["lb_loss"], rtol=1e-5)
    np.testing.assert_allclose(aux["compute_loss"].item(), d["compute_loss"], rtol=1e-5)
