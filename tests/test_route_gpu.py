"""Routing kernel: bit-exact against the oracle's stable sort / histogram /
rounded cumsums (the algorithm of fused_route, fused_cumsum.py:84-171)."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def _sel(A, E, seed, skew=False):
    rng = np.random.default_rng(seed)
    if skew:
        p = 1.0 / np.arange(1, E + 1) ** 1.1
        p /= p.sum()
        return rng.choice(E, size=A, p=p).astype(np.int64)
    return rng.integers(0, E, size=A).astype(np.int64)


ROUTE_CASES = [
    (0, 4, 64, "up", False),
    (1, 4, 64, "up", False),
    (32, 4, 64, "up", False),
    (64, 8, 128, "up", False),
    (16384, 16, 64, "up", False),
    (131072, 64, 64, "up", True),
    (524288, 128, 64, "up", True),
    (5000, 256, 16, "up", True),
    (4096, 8, 128, "down", False),
    (4096, 8, 128, "nearest", False),
    (777, 7, 32, "nearest", True),
    (3000, 1, 64, "up", False),
    # the multi-block path (past the single-CTA bound) in every rounding mode
    (6145, 8, 64, "up", False),
    (16384, 16, 64, "down", True),
    (10000, 7, 32, "nearest", True),
    (65536, 64, 128, "down", False),
]


@pytest.mark.parametrize("A,E,bs,rounding,skew", ROUTE_CASES)
@pytest.mark.parametrize("sel_dtype", [torch.int64, torch.int32])
def test_route_bit_exact(A, E, bs, rounding, skew, sel_dtype, device):
    from moe_b200.kernels import _ops

    sel_np = _sel(A, E, seed=A + E, skew=skew)
    ref = orc.fused_route(sel_np, E, bs, rounding)
    sel = torch.from_numpy(sel_np).to(device=device, dtype=sel_dtype)
    r = _ops.route(sel, E, bs, rounding)
    torch.cuda.synchronize()
    _ops.check_device_status(device)
    kept = int(ref["bins"][-1]) if E else 0
    np.testing.assert_array_equal(r.bin_ids[:kept].cpu().numpy(), ref["bin_ids"])
    np.testing.assert_array_equal(r.indices[:kept].cpu().numpy(), ref["indices"])
    for k in ("tokens_per_expert", "bins", "padded_bins"):
        np.testing.assert_array_equal(getattr(r, k).cpu().numpy(), ref[k])
    off = np.concatenate([[0], ref["padded_bins"]]).astype(np.int32)
    np.testing.assert_array_equal(r.expert_token_offsets.cpu().numpy(), off)
    P = int(off[-1])
    r2a, a2r = orc.row_maps(ref["indices"], ref["bin_ids"], ref["bins"], ref["padded_bins"], A)
    np.testing.assert_array_equal(r.row_to_assignment[:P].cpu().numpy(), r2a)
    if A:
        np.testing.assert_array_equal(r.assignment_to_row[:A].cpu().numpy(), a2r)


def test_route_rejects_bad_expert_ids(device):
    from moe_b200.kernels import _ops
    from moe_b200._lib import MoEKernelError

    sel = torch.tensor([0, 1, 9, 2], device=device)
    _ops.route(sel, 4, 16)
    torch.cuda.synchronize()
    with pytest.raises(MoEKernelError):
        _ops.check_device_status(device)
