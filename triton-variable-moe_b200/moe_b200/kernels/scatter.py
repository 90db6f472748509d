"""Padded scatter: un-permute expert rows and combine the top-k copies of a token.

Drop-in for triton_moe/kernels/scatter.py (padded_scatter :72-135,
PaddedScatterOp :138-176, padded_scatter_autograd :179-189).  The sm_100a
combine kernel reads each token's k rows through the inverse row map and sums
the weighted, storage-rounded products in fp32 in one pass, so the
reference's [T, k, H] temporary and its separate .sum(1) disappear.
"""

from __future__ import annotations

import torch
from torch.amp import custom_bwd, custom_fwd
from torch.autograd.function import once_differentiable

from . import _ops


@torch.compiler.disable
def padded_scatter(
    x: torch.Tensor,
    indices: torch.Tensor,
    bin_ids: torch.Tensor,
    weights: torch.Tensor,
    bins: torch.Tensor,
    padded_bins: torch.Tensor,
    top_k: int,
) -> torch.Tensor:
    """Scatter with padding (megablocks.ops.padded_scatter interface).

    Args:
        x: [padded_bins[-1], hidden] rows in padded expert order.
        weights: [num_tokens * top_k] routing weights indexed by assignment.

    Returns:
        [num_tokens, hidden]: out[t] = sum_j weights[t*k+j] * x[row(t, j)].
    """
    total_padded, hidden = x.shape
    num_tokens = len(weights) // top_k
    if len(indices) == 0:
        return torch.zeros(num_tokens, hidden, device=x.device, dtype=x.dtype)
    _, a2r = _ops.build_row_map(indices, bin_ids, bins, padded_bins, total_padded,
                                num_tokens * top_k, want_row_to_assignment=False)
    return _ops.combine(x, a2r, num_tokens, top_k, weights=weights.to(x.dtype))


class PaddedScatterOp(torch.autograd.Function):
    """Autograd function for padded_scatter.

    Backward is a weighted padded gather of the output gradient; like the
    reference (scatter.py:160-176) it returns no gradient for the weights.
    """

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, x, indices, bin_ids, weights, bins, padded_bins, top_k):
        ctx.save_for_backward(indices, bin_ids, weights, bins, padded_bins)
        ctx.top_k = top_k
        return padded_scatter(x, indices, bin_ids, weights, bins, padded_bins, top_k)

    @staticmethod
    @custom_bwd(device_type="cuda")
    @once_differentiable
    def backward(ctx, grad_output):
        from .gather import _weighted_padded_gather

        indices, bin_ids, weights, bins, padded_bins = ctx.saved_tensors
        grad_x = _weighted_padded_gather(grad_output, indices, bin_ids, weights, bins,
                                         padded_bins, ctx.top_k)
        return grad_x, None, None, None, None, None, None


def padded_scatter_autograd(x, indices, bin_ids, weights, bins, padded_bins, top_k):
    """Padded scatter with autograd support."""
    return PaddedScatterOp.apply(x, indices, bin_ids, weights, bins, padded_bins, top_k)
