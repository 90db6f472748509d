"""Routing: sort + histogram + rounded cumsums in one sm_100a routing pipeline.

Drop-in for triton_moe/kernels/fused_cumsum.py:84-171 (`fused_route`).  The
histogram, both inclusive cumsums, the rounding modes and the stable counting
sort all run on the device; for "down"/"nearest" rounding the dropped
assignments are compacted on the device as well, so only the final length of
the returned tensors needs a host read (the reference reads much more).
"""

from __future__ import annotations

import torch

from . import _ops


@torch.compiler.disable
def fused_route(
    selected_experts: torch.Tensor,
    num_experts: int,
    block_size: int = 128,
    rounding: str = "up",
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Stable sort of expert assignments plus per-expert bins.

    Args:
        selected_experts: [num_assignments] int32/int64 expert ids (token-major
            flattening of the top-k choice).
        num_experts: number of experts (at most 256).
        block_size: padding / rounding granularity.
        rounding: "up" (dropless), "down" or "nearest".

    Returns:
        (bin_ids, indices, tokens_per_expert, bins, padded_bins), all int32:
        the sorted expert ids, the stable argsort, the histogram, the
        inclusive cumsum of kept counts and of rounded counts.
    """
    assert selected_experts.is_cuda, "Input must be on CUDA"
    assert rounding in ("up", "down", "nearest"), f"Invalid rounding mode: {rounding}"
    r = _ops.route(selected_experts, num_experts, block_size, rounding, want_rows=False)
    if rounding == "up":
        return r.bin_ids, r.indices, r.tokens_per_expert, r.bins, r.padded_bins
    kept = int(r.bins[-1].item()) if num_experts > 0 else 0
    return r.bin_ids[:kept], r.indices[:kept], r.tokens_per_expert, r.bins, r.padded_bins
