"""Padded gather: permute tokens into expert-contiguous, block-padded rows.

Drop-in for triton_moe/kernels/gather.py (padded_gather :63-116,
_weighted_padded_gather :177-218, PaddedGatherOp :221-265,
padded_gather_autograd :268-277).  The sm_100a kernel walks padded rows (one
warp per row, 128-bit loads/stores) and writes padding rows as zeros itself,
so no zero-fill pass precedes it.
"""

from __future__ import annotations

import torch
from torch.amp import custom_bwd, custom_fwd
from torch.autograd.function import once_differentiable

from . import _ops


def _row_map(indices, bin_ids, bins, padded_bins, total_padded, num_assignments):
    r2a, _ = _ops.build_row_map(indices, bin_ids, bins, padded_bins, total_padded,
                                num_assignments, want_assignment_to_row=False)
    return r2a


@torch.compiler.disable
def padded_gather(
    x: torch.Tensor,
    indices: torch.Tensor,
    bin_ids: torch.Tensor,
    bins: torch.Tensor,
    padded_bins: torch.Tensor,
    top_k: int,
) -> torch.Tensor:
    """Gather with padding (megablocks.ops.padded_gather interface).

    Returns [padded_bins[-1], hidden] with zeros in the padding slots.
    """
    num_tokens, hidden = x.shape
    total_padded = int(padded_bins[-1].item()) if padded_bins.numel() else 0
    if len(indices) == 0 or total_padded == 0:
        return torch.zeros(total_padded, hidden, device=x.device, dtype=x.dtype)
    r2a = _row_map(indices, bin_ids, bins, padded_bins, total_padded, num_tokens * top_k)
    return _ops.gather(x, r2a, top_k, total_padded)


@torch.compiler.disable
def _weighted_padded_gather(
    x: torch.Tensor,
    indices: torch.Tensor,
    bin_ids: torch.Tensor,
    weights: torch.Tensor,
    bins: torch.Tensor,
    padded_bins: torch.Tensor,
    top_k: int,
) -> torch.Tensor:
    """padded_gather with each row multiplied by weights[assignment] (scatter backward)."""
    num_tokens, hidden = x.shape
    total_padded = int(padded_bins[-1].item()) if padded_bins.numel() else 0
    if len(indices) == 0 or total_padded == 0:
        return torch.zeros(total_padded, hidden, device=x.device, dtype=x.dtype)
    r2a = _row_map(indices, bin_ids, bins, padded_bins, total_padded, num_tokens * top_k)
    return _ops.gather(x, r2a, top_k, total_padded, weights=weights)


class PaddedGatherOp(torch.autograd.Function):
    """Autograd function for padded_gather (backward = unit-weight scatter)."""

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, x, indices, bin_ids, bins, padded_bins, top_k):
        ctx.save_for_backward(indices, bin_ids, bins, padded_bins)
        ctx.top_k = top_k
        ctx.num_tokens = x.shape[0]
        return padded_gather(x, indices, bin_ids, bins, padded_bins, top_k)

    @staticmethod
    @custom_bwd(device_type="cuda")
    @once_differentiable
    def backward(ctx, grad_output):
        from .scatter import padded_scatter

        indices, bin_ids, bins, padded_bins = ctx.saved_tensors
        weights = torch.ones(ctx.num_tokens * ctx.top_k, device=grad_output.device,
                             dtype=grad_output.dtype)
        grad_x = padded_scatter(grad_output, indices, bin_ids, weights, bins, padded_bins,
                                ctx.top_k)
        return grad_x, None, None, None, None, None


def padded_gather_autograd(x, indices, bin_ids, bins, padded_bins, top_k):
    """Padded gather with autograd support."""
    return PaddedGatherOp.apply(x, indices, bin_ids, bins, padded_bins, top_k)
