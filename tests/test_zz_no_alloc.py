"""moe_route_no_alloc: routing for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc: a plain C/FFI caller that
only holds the buffers it was given, or a runtime whose own pool or caching
allocator already owns the GPU's memory.  moe_route_no_alloc serves them by
keeping its histogram scratch in a fixed device array inside the library
instead of a caller-provided workspace.

This test calls it through the C ABI and checks that it produces exactly the
outputs of moe_route (integer results: bit-exact) on two calls in a row with
different problems, so that contents left in the shared array by the first
call cannot leak into the second.  The file is named to be collected last.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call_no_alloc(sel: torch.Tensor, E: int, bs: int, rounding: int):
    from moe_b200._lib import check, lib

    dev = sel.device
    A = sel.numel()
    cap = A + E * (bs - 1)
    i32 = dict(dtype=torch.int32, device=dev)
    out = dict(
        bin_ids=torch.full((max(A, 1),), -7, **i32),
        indices=torch.full((max(A, 1),), -7, **i32),
        tokens_per_expert=torch.full((E,), -7, **i32),
        bins=torch.full((E,), -7, **i32),
        padded_bins=torch.full((E,), -7, **i32),
        expert_token_offsets=torch.full((E + 1,), -7, **i32),
        padded_tokens_per_expert=torch.full((E,), -7, **i32),
        row_to_assignment=torch.full((cap,), -7, **i32),
        assignment_to_row=torch.full((max(A, 1),), -7, **i32),
    )
    status = torch.zeros(1, **i32)
    rc = lib.moe_route_no_alloc(
        sel.data_ptr(), 1 if sel.dtype == torch.int64 else 0, A, E, bs, rounding,
        out["bin_ids"].data_ptr(), out["indices"].data_ptr(), out["tokens_per_expert"].data_ptr(),
        out["bins"].data_ptr(), out["padded_bins"].data_ptr(),
        out["expert_token_offsets"].data_ptr(), out["padded_tokens_per_expert"].data_ptr(),
        out["row_to_assignment"].data_ptr(), cap, out["assignment_to_row"].data_ptr(),
        status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream,
    )
    check(rc, "moe_route_no_alloc")
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 0
    return out


def _check_against_moe_route(sel: torch.Tensor, E: int, bs: int):
    from moe_b200.kernels import _ops

    got = _call_no_alloc(sel, E, bs, 0)
    ref = _ops.route(sel, E, bs, "up")
    torch.cuda.synchronize()
    A = sel.numel()
    P = int(ref.expert_token_offsets[-1].item())
    pairs = [
        ("bin_ids", ref.bin_ids[:A]), ("indices", ref.indices[:A]),
        ("tokens_per_expert", ref.tokens_per_expert), ("bins", ref.bins),
        ("padded_bins", ref.padded_bins), ("expert_token_offsets", ref.expert_token_offsets),
        ("padded_tokens_per_expert", ref.padded_tokens_per_expert),
        ("row_to_assignment", ref.row_to_assignment[:P]),
        ("assignment_to_row", ref.assignment_to_row[:A]),
    ]
    for name, want in pairs:
        n = want.numel()
        np.testing.assert_array_equal(got[name][:n].cpu().numpy(), want.cpu().numpy(),
                                      err_msg=name)


def test_no_alloc_route_matches_route_twice(device):
    g = torch.Generator(device="cpu").manual_seed(5)
    # first call: the largest scratch the entry point supports (256 units x 256
    # experts): 256 * 1184 assignments make units of 1184, exactly 256 of them
    sel1 = torch.randint(0, 256, (256 * 1184,), generator=g).to(device)
    _check_against_moe_route(sel1, 256, 64)
    # second call, different problem (int32 ids, skewed, fewer experts)
    p = 1.0 / torch.arange(1, 17, dtype=torch.float64) ** 1.1
    sel2 = torch.multinomial(p / p.sum(), 20_000, replacement=True, generator=g).to(torch.int32)
    _check_against_moe_route(sel2.to(device), 16, 128)


def test_no_alloc_route_rejects_too_many_experts(device):
    from moe_b200._lib import MoEKernelError

    sel = torch.zeros(10, dtype=torch.int64, device=device)
    with pytest.raises(MoEKernelError):
        _call_no_alloc(sel, 300, 16, 0)
