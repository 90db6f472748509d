"""SwiGLU up projection (activation="swiglu") on the GPU.

* Forward against the reference's own kernel (golden vectors made under the
  Triton interpreter, fp32) and the oracle in bf16: out = silu(gate) * up with
  each expert's w1 columns laid out gate block then up block, pre_act = gate.
  Tolerance: the bf16 bound |a - b| <= 1e-2 * max|b| + 2e-2 * |b|.
* The stored gate / up projections against torch fp32, both N tiles, ragged
  widths (not multiples of the tile).
* Backward: the reference's swiglu backward is a placeholder, so gradients are
  checked against torch autograd of the same expression (fp32 math on the same
  bf16 inputs), same tolerance.
"""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from tests.goldens import load
from tests.test_api_gpu import assert_close_scaled

pytestmark = pytest.mark.gpu

SWIGLU = load("swiglu")
BF = torch.bfloat16


def _meta(widths, counts, device):
    i32 = dict(dtype=torch.int32, device=device)
    tok = torch.tensor([0] + list(np.cumsum(counts)), **i32)
    woff = torch.tensor([0] + list(np.cumsum([2 * w for w in widths])), **i32)
    return tok, woff, torch.tensor(widths, **i32), torch.tensor(counts, **i32)


@pytest.mark.parametrize("case", sorted(SWIGLU))
def test_swiglu_forward_matches_reference(case, device):
    from moe_b200.kernels import grouped_gemm_up

    d = SWIGLU[case]
    maxw = int(d["widths"].max())
    q = {n: orc.round_bf16(d[n]) for n in ("x", "w1")}
    args = [torch.from_numpy(d[n]).to(device) for n in ("tok_off", "w_off")]
    widths = torch.from_numpy(d["widths"].astype(np.int32)).to(device)
    tpe = torch.from_numpy(d["counts"].astype(np.int32)).to(device)
    x = torch.from_numpy(q["x"]).to(device, BF)
    w1 = torch.from_numpy(q["w1"]).to(device, BF)
    out, pre = grouped_gemm_up(x, w1, *args, widths, tpe, maxw, activation="swiglu",
                               save_pre_act=True)
    assert_close_scaled(out.float().cpu(), d["out"], "swiglu out vs reference")
    assert_close_scaled(pre.float().cpu(), d["pre"], "swiglu gate vs reference")
    o_out, o_pre = orc.grouped_gemm_up(q["x"], q["w1"], d["tok_off"], d["w_off"], maxw, "swiglu",
                                       dtype="bf16")
    assert_close_scaled(out.float().cpu(), o_out, "swiglu out vs oracle")
    assert_close_scaled(pre.float().cpu(), o_pre, "swiglu gate vs oracle")


@pytest.mark.parametrize("tile_n", [128, 256])
@pytest.mark.parametrize("widths,counts,H", [([512, 256, 128], [300, 17, 0], 256),
                                             ([48, 80, 208], [64, 129, 40], 128)])
def test_swiglu_gate_up_outputs(tile_n, widths, counts, H, device):
    from moe_b200.kernels import _ops

    g = torch.Generator(device="cpu").manual_seed(5)
    tok, woff, wid, tpe = _meta(widths, counts, device)
    P, TW, maxw = int(tok[-1]), int(woff[-1]), max(widths)
    x = torch.randn(max(P, 1), H, generator=g).to(device, BF)
    w1 = (torch.randn(H, TW, generator=g) / H ** 0.5).to(device, BF)
    out = torch.zeros(max(P, 1), maxw, dtype=BF, device=device)
    gate, up = torch.zeros_like(out), torch.zeros_like(out)
    _ops.gemm_up_swiglu(x, w1, tok, woff, tpe, len(widths), out, gate=gate, up=up, tile_n=tile_n)
    torch.cuda.synchronize()
    _ops.check_device_status(device)
    wo = [int(v) for v in woff.tolist()]
    to = [int(v) for v in tok.tolist()]
    for e, w in enumerate(widths):
        r0, r1 = to[e], to[e + 1]
        if r1 == r0:
            continue
        zg = x[r0:r1].float() @ w1[:, wo[e]:wo[e] + w].float()
        zu = x[r0:r1].float() @ w1[:, wo[e] + w:wo[e] + 2 * w].float()
        assert_close_scaled(gate[r0:r1, :w].cpu(), zg.cpu().numpy(), f"gate e{e}")
        assert_close_scaled(up[r0:r1, :w].cpu(), zu.cpu().numpy(), f"up e{e}")
        assert_close_scaled(out[r0:r1, :w].cpu(), (torch.nn.functional.silu(zg) * zu).cpu().numpy(),
                            f"out e{e}")
        assert (out[r0:r1, w:] == 0).all(), "columns beyond the expert width stay untouched"


@pytest.mark.parametrize("widths,counts,H", [([64, 32, 48], [64, 32, 48], 48),
                                             ([256, 128], [208, 80], 256)])
def test_swiglu_backward_matches_autograd(widths, counts, H, device):
    from moe_b200.kernels import grouped_gemm_up_autograd, grouped_gemm_up_backward

    g = torch.Generator(device="cpu").manual_seed(7)
    tok, woff, wid, tpe = _meta(widths, counts, device)
    P, TW, maxw = int(tok[-1]), int(woff[-1]), max(widths)
    x = torch.randn(P, H, generator=g).to(device, BF).requires_grad_()
    w1 = (torch.randn(H, TW, generator=g) / H ** 0.5).to(device, BF).requires_grad_()
    gout = torch.randn(P, maxw, generator=g).to(device, BF)
    out = grouped_gemm_up_autograd(x, w1, tok, woff, wid, tpe, maxw, H, activation="swiglu")
    out.backward(gout)
    from moe_b200.kernels import _ops as ops_

    ops_.check_device_status(device)  # row counts here are multiples of 16, as required
    # torch autograd of the same expression, fp32 math on the same bf16 inputs
    xr = x.detach().float().requires_grad_()
    wr = w1.detach().float().requires_grad_()
    to, wo = [int(v) for v in tok.tolist()], [int(v) for v in woff.tolist()]
    loss = 0.0
    for e, w in enumerate(widths):
        r0, r1 = to[e], to[e + 1]
        zg = xr[r0:r1] @ wr[:, wo[e]:wo[e] + w]
        zu = xr[r0:r1] @ wr[:, wo[e] + w:wo[e] + 2 * w]
        loss = loss + (torch.nn.functional.silu(zg) * zu * gout[r0:r1, :w].float()).sum()
    loss.backward()
    assert_close_scaled(x.grad.float().cpu(), xr.grad.cpu().numpy(), "swiglu dX")
    assert_close_scaled(w1.grad.float().cpu(), wr.grad.cpu().numpy(), "swiglu dW1")
    # the functional backward without the saved up projection recomputes it
    gate = torch.zeros(P, maxw, dtype=BF, device=device)
    from moe_b200.kernels import _ops

    _ops.gemm_up_swiglu(x.detach(), w1.detach(), tok, woff, tpe, len(widths),
                        torch.zeros_like(gate), gate=gate)
    gx2, gw2 = grouped_gemm_up_backward(gout, x.detach(), w1.detach(), gate, tok, woff, wid, tpe,
                                        H, "swiglu")
    assert torch.equal(gx2, x.grad) and torch.equal(gw2, w1.grad)
