"""A device-side wait that runs out returns an error status and leaves the
context usable.

The fused up + down launch (moe_grouped_gemm_up_down) makes every down tile
wait, bounded in time, until the up tiles of its 128-row block have stored
their part of the intermediate; the block's counter word says how many have.
Here the counters start far below zero, so no block ever looks complete: with
the wait limit set to 1 ms (moe_set_wait_timeout_ns) every waiting tile gives
up, the launch ends with MOE_ERR_TIMEOUT in its status word and returns
(copies and MMAs in flight drained, tensor memory released).  The next
launch on the same device, with the default limit and zeroed counters, must
give exactly the separate up + down launches' results.  Nothing here faults
or hangs the GPU: the only wait that runs out is a bounded poll of a counter.
"""

import pytest
import torch

from tests.test_grouped_gemm_gpu import make_problem

pytestmark = pytest.mark.gpu

MOE_ERR_TIMEOUT = -4


def _launch(t, m, dep, status, h, pre, y, H):
    from moe_b200 import _lib

    return _lib.lib.moe_grouped_gemm_up_down(
        t["x"].data_ptr(), m["rows"], t["x"].stride(0), t["w1"].data_ptr(), t["w2"].data_ptr(),
        H, m["TW"], m["tok_off"].data_ptr(), m["w_off"].data_ptr(), m["tpe"].data_ptr(), m["E"],
        h.data_ptr(), pre.data_ptr(), h.stride(0), y.data_ptr(), y.stride(0), dep.data_ptr(),
        dep.numel(), 0, 256, 256, status.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_row_block_wait_times_out_then_next_launch_is_correct(device):
    from moe_b200 import _lib
    from moe_b200.kernels import _ops

    widths, counts, H = [256, 128, 256], [300, 70, 129], 256
    t, m = make_problem(widths, counts, H, 64, device=device, seed=3)
    for k in ("x", "w1", "w2"):
        t[k] = t[k].to(device)
    words = int(_lib.lib.moe_up_down_dep_words(m["rows"], m["E"]))
    status = torch.zeros(1, dtype=torch.int32, device=device)
    h = torch.zeros(m["rows"], m["maxw"], dtype=torch.bfloat16, device=device)
    pre, y = torch.zeros_like(h), torch.zeros(m["rows"], H, dtype=torch.bfloat16, device=device)

    # 1. counters that never reach their target: every down tile's wait runs out
    dep = torch.full((words,), -(1 << 30), dtype=torch.int32, device=device)
    prev = _lib.lib.moe_set_wait_timeout_ns(1_000_000)  # 1 ms
    try:
        rc = _launch(t, m, dep, status, h, pre, y, H)
        torch.cuda.synchronize()  # the launch returned on its own
    finally:
        _lib.lib.moe_set_wait_timeout_ns(0)
    assert rc == 0
    assert int(status.item()) == MOE_ERR_TIMEOUT
    assert prev == 2_000_000_000

    # 2. the next launch on the same device: default limit, zeroed counters
    status.zero_()
    dep = torch.zeros(words, dtype=torch.int32, device=device)
    h.zero_(), pre.zero_(), y.zero_()
    assert _launch(t, m, dep, status, h, pre, y, H) == 0
    args = (m["tok_off"], m["w_off"], m["tpe"], m["E"])
    h2, pre2 = torch.zeros_like(h), torch.zeros_like(h)
    _ops.gemm_up(t["x"], t["w1"], *args, "relu_squared", h2, pre2, tile_n=256)
    y2 = torch.zeros_like(y)
    _ops.gemm_down(h2, t["w2"], *args, y2, tile_n=256)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(h, h2) and torch.equal(pre, pre2) and torch.equal(y, y2)
    assert int(dep.abs().sum().item()) == 0  # the counters are back at zero
    _ops.check_device_status(device)
