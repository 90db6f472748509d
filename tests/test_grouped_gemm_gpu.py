"""Grouped GEMM kernels (tcgen05) against a plain PyTorch fp32 reference.

Each of the six MoE GEMMs is checked expert by expert on random grouped
problems, including experts with no rows, widths that are not multiples of
the 64-wide k-block, both N tiles, and the fused relu^2 / relu^2-derivative
epilogues.  Tolerance (bf16 storage, fp32 accumulation): |a-b| <= 1e-2 +
2e-2 |b| (bf16 results against an fp32 reference).
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 1e-2
PAIR = 0x200  # tile_n flag (MOE_TILE_PAIR): 256-row tiles on 2-CTA clusters
TILES = [128, 256, 128 | PAIR, 256 | PAIR]


def assert_close(a, b, what):
    a = a.float()
    b = b.float()
    bad = (a - b).abs() > ATOL + RTOL * b.abs()
    if bad.any():
        i = bad.nonzero()[0].tolist()
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.numel()} mismatches, first at {i}: "
            f"got {a[tuple(i)].item()} want {b[tuple(i)].item()}; max abs err "
            f"{(a - b).abs().max().item():.3e}"
        )


def make_problem(widths, counts, H, bs, dtype=torch.bfloat16, seed=0, device="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    E = len(widths)
    padded = [math.ceil(c / bs) * bs for c in counts]
    tok_off = [0]
    for p in padded:
        tok_off.append(tok_off[-1] + p)
    w_off = [0]
    for w in widths:
        w_off.append(w_off[-1] + w)
    P, TW, maxw = tok_off[-1], w_off[-1], max(widths)
    rows = max(P, 1)
    x = torch.randn(rows, H, generator=g).to(dtype)
    w1 = (torch.randn(H, TW, generator=g) / math.sqrt(H)).to(dtype)
    w2 = (torch.randn(TW, H, generator=g) / math.sqrt(maxw)).to(dtype)
    gy = torch.randn(rows, H, generator=g).to(dtype)
    ga = torch.randn(rows, maxw, generator=g).to(dtype)
    pre = torch.relu(torch.randn(rows, maxw, generator=g)).to(dtype)
    i32 = dict(dtype=torch.int32, device=device)
    meta = dict(
        tok_off=torch.tensor(tok_off, **i32),
        w_off=torch.tensor(w_off, **i32),
        tpe=torch.tensor(padded, **i32),
        E=E,
        tok=tok_off,
        wo=w_off,
        P=P,
        rows=rows,
        maxw=maxw,
        TW=TW,
    )
    t = {k: v.to(device) for k, v in dict(x=x, w1=w1, w2=w2, gy=gy, ga=ga, pre=pre).items()}
    return t, meta


CASES = [
    # widths, counts, H, block
    ([128, 256, 512, 128], [100, 0, 300, 64], 256, 64),
    ([512, 512], [1000, 37], 768, 64),
    ([64, 192, 320], [5, 129, 64], 128, 128),
    ([48, 80, 16], [16, 40, 70], 64, 16),  # K tails that are not a multiple of 64
    ([256] * 8, [130] * 8, 256, 128),
]


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
@pytest.mark.parametrize("tile_n", TILES)
def test_up_forward(case, tile_n, device):
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, device=device)
    out = torch.zeros(m["rows"], m["maxw"], dtype=torch.bfloat16, device=device)
    pre = torch.zeros_like(out)
    _ops.gemm_up(t["x"], t["w1"], m["tok_off"], m["w_off"], m["tpe"], m["E"], "relu_squared",
                 out, pre, tile_n=tile_n)
    torch.cuda.synchronize()
    _ops.check_device_status(device)
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        if r1 == r0:
            continue
        z = t["x"][r0:r1].float() @ t["w1"][:, c0:c1].float()
        assert_close(pre[r0:r1, : c1 - c0], torch.relu(z), f"pre e{e}")
        assert_close(out[r0:r1, : c1 - c0], torch.relu(z) ** 2, f"out e{e}")
        assert (out[r0:r1, c1 - c0:] == 0).all(), "columns beyond the expert width must be untouched"


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
def test_up_forward_no_activation(case, device):
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, device=device, seed=1)
    out = torch.zeros(m["rows"], m["maxw"], dtype=torch.bfloat16, device=device)
    _ops.gemm_up(t["x"], t["w1"], m["tok_off"], m["w_off"], m["tpe"], m["E"], "none", out)
    torch.cuda.synchronize()
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        if r1 > r0:
            z = t["x"][r0:r1].float() @ t["w1"][:, c0:c1].float()
            assert_close(out[r0:r1, : c1 - c0], z, f"out e{e}")


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
@pytest.mark.parametrize("tile_n", TILES)
def test_down_forward(case, tile_n, device):
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, device=device, seed=2)
    y = torch.zeros(m["rows"], H, dtype=torch.bfloat16, device=device)
    _ops.gemm_down(t["ga"], t["w2"], m["tok_off"], m["w_off"], m["tpe"], m["E"], y, tile_n=tile_n)
    torch.cuda.synchronize()
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        if r1 > r0:
            ref = t["ga"][r0:r1, : c1 - c0].float() @ t["w2"][c0:c1].float()
            assert_close(y[r0:r1], ref, f"y e{e}")


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("tile_n", [0, 128 | PAIR])
def test_down_dinter(case, fused, tile_n, device):
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, device=device, seed=3)
    out = torch.zeros(m["rows"], m["maxw"], dtype=torch.bfloat16, device=device)
    _ops.gemm_down_dinter(t["gy"], t["w2"], m["tok_off"], m["w_off"], m["tpe"], m["E"], out,
                          pre_act=t["pre"] if fused else None, tile_n=tile_n)
    torch.cuda.synchronize()
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        if r1 == r0:
            continue
        g = t["gy"][r0:r1].float() @ t["w2"][c0:c1].float().T
        if fused:
            p = t["pre"][r0:r1, : c1 - c0].float()
            g = torch.where(p > 0, g.bfloat16().float() * 2.0 * p, torch.zeros_like(p))
        assert_close(out[r0:r1, : c1 - c0], g, f"dinter e{e}")


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
@pytest.mark.parametrize("tile_n", TILES)
def test_up_dx(case, tile_n, device):
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, device=device, seed=4)
    gx = torch.zeros(m["rows"], H, dtype=torch.bfloat16, device=device)
    _ops.gemm_up_dx(t["ga"], t["w1"], m["tok_off"], m["w_off"], m["tpe"], m["E"], gx, tile_n=tile_n)
    torch.cuda.synchronize()
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        if r1 > r0:
            ref = t["ga"][r0:r1, : c1 - c0].float() @ t["w1"][:, c0:c1].float().T
            assert_close(gx[r0:r1], ref, f"gx e{e}")


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
@pytest.mark.parametrize("tile_n", TILES)
def test_up_dw(case, tile_n, device):
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, device=device, seed=5)
    gw1 = torch.full((H, m["TW"]), 7.0, dtype=torch.bfloat16, device=device)
    _ops.gemm_up_dw(t["x"], t["ga"], m["tok_off"], m["w_off"], m["E"], gw1, tile_n=tile_n)
    torch.cuda.synchronize()
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        ref = t["x"][r0:r1].float().T @ t["ga"][r0:r1, : c1 - c0].float()
        assert_close(gw1[:, c0:c1], ref, f"gw1 e{e}")  # experts with no rows -> zeros


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
@pytest.mark.parametrize("tile_n", TILES)
def test_down_dw(case, tile_n, device):
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, device=device, seed=6)
    gw2 = torch.full((m["TW"], H), 7.0, dtype=torch.bfloat16, device=device)
    _ops.gemm_down_dw(t["ga"], t["gy"], m["tok_off"], m["w_off"], m["E"], gw2, tile_n=tile_n)
    torch.cuda.synchronize()
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        ref = t["ga"][r0:r1, : c1 - c0].float().T @ t["gy"][r0:r1].float()
        assert_close(gw2[c0:c1], ref, f"gw2 e{e}")


def test_fp16_up(device):
    from moe_b200.kernels import _ops

    t, m = make_problem([128, 256], [64, 200], 256, 64, dtype=torch.float16, device=device, seed=7)
    out = torch.zeros(m["rows"], m["maxw"], dtype=torch.float16, device=device)
    _ops.gemm_up(t["x"], t["w1"], m["tok_off"], m["w_off"], m["tpe"], m["E"], "none", out)
    torch.cuda.synchronize()
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        ref = t["x"][r0:r1].float() @ t["w1"][:, c0:c1].float()
        assert_close(out[r0:r1, : c1 - c0], ref, f"fp16 e{e}")


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
@pytest.mark.parametrize("pair", [0, PAIR])
def test_fused_backward_launches(case, pair, device):
    """The two-problem launches (dIntermediate+dW2, dX+dW1) give the same
    results as the single-problem launches (128-row or paired 256-row tiles)."""
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, device=device, seed=8)
    args = (m["tok_off"], m["w_off"], m["tpe"], m["E"])
    dact = torch.zeros(m["rows"], m["maxw"], dtype=torch.bfloat16, device=device)
    gw2 = torch.full((m["TW"], H), 7.0, dtype=torch.bfloat16, device=device)
    _ops.gemm_down_backward(t["gy"], t["ga"], t["w2"], *args, dact, gw2, pre_act=t["pre"],
                            tile_n_width=128 | pair, tile_n_hidden=256 | pair)
    dact_ref = torch.zeros_like(dact)
    _ops.gemm_down_dinter(t["gy"], t["w2"], *args, dact_ref, pre_act=t["pre"], tile_n=128 | pair)
    gw2_ref = torch.zeros_like(gw2)
    _ops.gemm_down_dw(t["ga"], t["gy"], m["tok_off"], m["w_off"], m["E"], gw2_ref,
                      tile_n=256 | pair)
    torch.cuda.synchronize()
    assert torch.equal(dact, dact_ref)
    assert torch.equal(gw2, gw2_ref)
    gx = torch.zeros(m["rows"], H, dtype=torch.bfloat16, device=device)
    gw1 = torch.full((H, m["TW"]), 7.0, dtype=torch.bfloat16, device=device)
    _ops.gemm_up_backward(t["ga"], t["x"], t["w1"], *args, gx, gw1, tile_n_width=128 | pair,
                          tile_n_hidden=256 | pair)
    gx_ref = torch.zeros_like(gx)
    _ops.gemm_up_dx(t["ga"], t["w1"], *args, gx_ref, tile_n=256 | pair)
    gw1_ref = torch.zeros_like(gw1)
    _ops.gemm_up_dw(t["x"], t["ga"], m["tok_off"], m["w_off"], m["E"], gw1_ref,
                    tile_n=128 | pair)
    torch.cuda.synchronize()
    assert torch.equal(gx, gx_ref)
    assert torch.equal(gw1, gw1_ref)
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        ref = t["x"][r0:r1].float().T @ t["ga"][r0:r1, : c1 - c0].float()
        assert_close(gw1[:, c0:c1], ref, f"gw1 e{e}")


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
@pytest.mark.parametrize("tiles", [(128, 128), (256, 256), (128, 256)])
def test_fused_up_down_matches_separate_launches(case, tiles, device):
    """One launch of up (relu^2) + down with row-block dependencies gives exactly
    the two separate launches' results, and leaves its counters at zero."""
    from moe_b200.kernels import _ops

    widths, counts, H, bs = case
    t, m = make_problem(widths, counts, H, bs, device=device, seed=12)
    args = (m["tok_off"], m["w_off"], m["tpe"], m["E"])
    tw, th = tiles
    for rep in range(3):  # the counters are reused across launches
        h = torch.zeros(m["rows"], m["maxw"], dtype=torch.bfloat16, device=device)
        pre = torch.zeros_like(h)
        y = torch.zeros(m["rows"], H, dtype=torch.bfloat16, device=device)
        _ops.gemm_up_down(t["x"], t["w1"], t["w2"], *args, h, pre, y, tile_n_width=tw,
                          tile_n_hidden=th)
        h2 = torch.zeros_like(h)
        pre2 = torch.zeros_like(h)
        _ops.gemm_up(t["x"], t["w1"], *args, "relu_squared", h2, pre2, tile_n=tw)
        y2 = torch.zeros_like(y)
        _ops.gemm_down(h2, t["w2"], *args, y2, tile_n=th)
        torch.cuda.synchronize()
        _ops.check_device_status(device)
        assert torch.equal(h, h2) and torch.equal(pre, pre2)
        assert torch.equal(y, y2)
        dep = _ops.up_down_dep_buffer(device, m["rows"], m["E"])
        assert int(dep.abs().sum().item()) == 0


SKEWED = ([256] * 8, [2000, 700, 300, 100, 40, 10, 0, 5], 512, 64)


@pytest.mark.parametrize("ctas", [3, 7])
def test_ticket_schedule_backward_matches_round_robin(ctas, device):
    """With at least 8 tiles per CTA a launch takes its tiles by ticket from a
    per-stream counter (skewed routing makes the weight-gradient tiles' K very
    unequal).  Capping the grid forces that schedule at a small size; every
    output equals the round-robin launch of the full grid bit for bit, the
    counter is reused across launches, and dW1 matches the fp32 reference."""
    from moe_b200 import _lib
    from moe_b200.kernels import _ops

    widths, counts, H, bs = SKEWED
    t, m = make_problem(widths, counts, H, bs, device=device, seed=21)
    args = (m["tok_off"], m["w_off"], m["tpe"], m["E"])
    cap = _lib.tile_ctas(ctas)

    def run(extra):
        dact = torch.zeros(m["rows"], m["maxw"], dtype=torch.bfloat16, device=device)
        gw2 = torch.full((m["TW"], H), 7.0, dtype=torch.bfloat16, device=device)
        _ops.gemm_down_backward(t["gy"], t["ga"], t["w2"], *args, dact, gw2,
                                pre_act=t["pre"], tile_n_width=128 | extra,
                                tile_n_hidden=256 | extra)
        gx = torch.zeros(m["rows"], H, dtype=torch.bfloat16, device=device)
        gw1 = torch.full((H, m["TW"]), 7.0, dtype=torch.bfloat16, device=device)
        _ops.gemm_up_backward(t["ga"], t["x"], t["w1"], *args, gx, gw1,
                              tile_n_width=128 | extra, tile_n_hidden=256 | extra)
        torch.cuda.synchronize()
        _ops.check_device_status(device)
        return dact, gw2, gx, gw1

    want = run(0)
    for _rep in range(3):  # the ticket counter returns to zero after every launch
        for a, b in zip(run(cap), want):
            assert torch.equal(a, b)
    gw1 = want[3]
    for e in range(m["E"]):
        r0, r1, c0, c1 = m["tok"][e], m["tok"][e + 1], m["wo"][e], m["wo"][e + 1]
        ref = t["x"][r0:r1].float().T @ t["ga"][r0:r1, : c1 - c0].float()
        assert_close(gw1[:, c0:c1], ref, f"gw1 e{e}")


@pytest.mark.parametrize("ctas", [2, 5])
def test_ticket_schedule_fused_forward(ctas, device):
    """The fused up + down launch on a capped grid takes its tiles by ticket:
    every up tile is taken before any down tile, so a down tile waits only for
    up tiles that running blocks hold.  Same results as the separate launches."""
    from moe_b200 import _lib
    from moe_b200.kernels import _ops

    widths, counts, H, bs = SKEWED
    t, m = make_problem(widths, counts, H, bs, device=device, seed=22)
    args = (m["tok_off"], m["w_off"], m["tpe"], m["E"])
    cap = _lib.tile_ctas(ctas)
    h2 = torch.zeros(m["rows"], m["maxw"], dtype=torch.bfloat16, device=device)
    pre2 = torch.zeros_like(h2)
    _ops.gemm_up(t["x"], t["w1"], *args, "relu_squared", h2, pre2, tile_n=256)
    y2 = torch.zeros(m["rows"], H, dtype=torch.bfloat16, device=device)
    _ops.gemm_down(h2, t["w2"], *args, y2, tile_n=256)
    for _rep in range(2):
        h = torch.zeros_like(h2)
        pre = torch.zeros_like(h2)
        y = torch.zeros_like(y2)
        _ops.gemm_up_down(t["x"], t["w1"], t["w2"], *args, h, pre, y, tile_n_width=256 | cap,
                          tile_n_hidden=256 | cap)
        torch.cuda.synchronize()
        _ops.check_device_status(device)
        assert torch.equal(h, h2) and torch.equal(pre, pre2) and torch.equal(y, y2)
