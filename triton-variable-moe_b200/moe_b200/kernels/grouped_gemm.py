"""Grouped GEMMs for the MoE up/down projections on sm_100a tensor cores.

Drop-in for triton_moe/kernels/grouped_gemm.py: precompute_gather_map
(:104-149), grouped_gemm_up (:378-477), grouped_gemm_down (:586-651),
grouped_gemm_up_backward (:1165-1290), grouped_gemm_down_backward
(:1293-1390), GroupedGemmUp / GroupedGemmDown (:1393-1601) and the autograd
wrappers (:1604-1665).

All six GEMMs run on one persistent tcgen05 engine (csrc/grouped_gemm.cu):
operands arrive by TMA, the accumulator lives in tensor memory, and every CTA
derives each expert's tile geometry on the device from the offset arrays, so
no tile schedule or sparse topology is built on the host.

Layouts (as in the reference):
    w1: [hidden, total_expert_width]   experts concatenated along columns
    w2: [total_expert_width, hidden]   experts concatenated along rows
    intermediate: [total_tokens, max_expert_width]; expert e uses columns
        [0, w_e) of its rows, the other columns are zero.

Activations: "relu_squared", "none" and "swiglu".  For "swiglu" expert e's
w1 columns are its gate block then its up block (expert_weight_offsets step by
2 w_e, the reference's layout, grouped_gemm.py:296-358); the forward matches
the reference's (output silu(gate) * up, pre_act = gate).  The reference's
swiglu backward is an acknowledged placeholder (grouped_gemm.py:768-789,
930-942); here it is the true gradient: dgate = g * up * silu'(gate),
dup = g * silu(gate), then the usual dX / dW GEMMs over width 2 w_e.  The up
projection is kept by the autograd function, or recomputed when
grouped_gemm_up_backward is called without it.
"""

from __future__ import annotations

import torch
from torch.amp import custom_bwd, custom_fwd
from torch.autograd.function import once_differentiable

from . import _ops

_SUPPORTED_ACTIVATIONS = ("relu_squared", "none", "swiglu")


def _check_swiglu_layout(expert_weight_offsets, expert_widths) -> None:
    """The swiglu kernels take each expert's up block right after its gate block."""
    off = expert_weight_offsets.to(torch.int64)
    wid = expert_widths.to(torch.int64)
    if not torch.equal(off[1:] - off[:-1], 2 * wid):
        raise ValueError("swiglu: expert_weight_offsets must step by 2 * expert_widths "
                         "(each expert's gate columns, then its up columns)")


def _check_activation(activation: str) -> None:
    if activation not in _SUPPORTED_ACTIVATIONS:
        raise NotImplementedError(
            f"activation {activation!r} is not supported (supported: {_SUPPORTED_ACTIVATIONS})"
        )


def _gather_rows(x: torch.Tensor, gather_map: torch.Tensor, rows: int) -> torch.Tensor:
    """x[gather_map] for the fused-gather path (padding rows map to row 0, as the
    reference's USE_GATHER_MAP loads do)."""
    gm = gather_map.to(torch.int32).contiguous()
    return _ops.gather(x, gm, 1, rows)


@torch.compiler.disable
def precompute_gather_map(
    indices: torch.Tensor,
    bin_ids: torch.Tensor,
    bins: torch.Tensor,
    padded_bins: torch.Tensor,
    top_k: int,
) -> torch.Tensor:
    """Map gathered-space (padded) rows to original token rows; padding rows -> 0."""
    total_padded = int(padded_bins[-1].item()) if padded_bins.numel() else 0
    if len(indices) == 0 or total_padded == 0:
        return torch.zeros(total_padded, dtype=torch.int32, device=indices.device)
    r2a, _ = _ops.build_row_map(indices, bin_ids, bins, padded_bins, total_padded, 0,
                                want_assignment_to_row=False)
    return _ops.gather_map(r2a, total_padded, top_k)


@torch.compiler.disable
def grouped_gemm_up(
    x: torch.Tensor,
    w1: torch.Tensor,
    expert_token_offsets: torch.Tensor,
    expert_weight_offsets: torch.Tensor,
    expert_widths: torch.Tensor,
    tokens_per_expert: torch.Tensor,
    max_expert_width: int,
    activation: str = "relu_squared",
    save_pre_act: bool = False,
    gather_map: torch.Tensor | None = None,
):
    """Grouped up-projection with fused activation.

    Returns the activated intermediate [total_tokens, max_expert_width], or
    (output, pre_act) when save_pre_act (pre_act = relu(x @ W1) for relu^2).
    """
    _check_activation(activation)
    total_tokens = int(expert_token_offsets[-1].item())
    dtype = x.dtype
    out = torch.zeros(total_tokens, max_expert_width, device=x.device, dtype=dtype)
    pre = torch.zeros_like(out) if save_pre_act else None
    if total_tokens == 0:
        return (out, pre) if save_pre_act else out
    if activation == "swiglu":
        _check_swiglu_layout(expert_weight_offsets, expert_widths)
        if gather_map is not None:
            x = _gather_rows(x, gather_map, total_tokens)
        _ops.gemm_up_swiglu(x.contiguous(), w1.contiguous(), expert_token_offsets,
                            expert_weight_offsets, tokens_per_expert, len(expert_widths), out,
                            gate=pre)
        return (out, pre) if save_pre_act else out
    if gather_map is not None:
        x = _gather_rows(x, gather_map, total_tokens)
    _ops.gemm_up(x.contiguous(), w1.contiguous(), expert_token_offsets, expert_weight_offsets,
                 tokens_per_expert, len(expert_widths), activation, out,
                 pre if activation == "relu_squared" else None)
    if save_pre_act and activation == "none":
        pre.copy_(out)
    return (out, pre) if save_pre_act else out


@torch.compiler.disable
def grouped_gemm_down(
    intermediate: torch.Tensor,
    w2: torch.Tensor,
    expert_token_offsets: torch.Tensor,
    expert_weight_offsets: torch.Tensor,
    expert_widths: torch.Tensor,
    tokens_per_expert: torch.Tensor,
    hidden_size: int,
) -> torch.Tensor:
    """Grouped down-projection: out[rows_e] = intermediate[rows_e, :w_e] @ W2_e."""
    total_tokens = intermediate.shape[0]
    out = torch.zeros(total_tokens, hidden_size, device=intermediate.device,
                      dtype=intermediate.dtype)
    if total_tokens == 0:
        return out
    _ops.gemm_down(intermediate.contiguous(), w2.contiguous(), expert_token_offsets,
                   expert_weight_offsets, tokens_per_expert, len(expert_widths), out)
    return out


@torch.compiler.disable
def grouped_gemm_up_backward(
    grad_output: torch.Tensor,
    x: torch.Tensor,
    w1: torch.Tensor,
    pre_act: torch.Tensor,
    expert_token_offsets: torch.Tensor,
    expert_weight_offsets: torch.Tensor,
    expert_widths: torch.Tensor,
    tokens_per_expert: torch.Tensor,
    hidden_size: int,
    activation: str = "relu_squared",
    gather_map: torch.Tensor | None = None,
    up_act: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gradients of grouped_gemm_up: (grad_x in gathered space, grad_w1).

    For "swiglu", pre_act is the gate projection and up_act the up projection
    (recomputed when not given)."""
    _check_activation(activation)
    total_tokens = int(expert_token_offsets[-1].item())
    dtype = x.dtype
    grad_x = torch.zeros(total_tokens, hidden_size, device=x.device, dtype=dtype)
    grad_w1 = torch.zeros_like(w1)
    if total_tokens == 0:
        return grad_x, grad_w1
    g = grad_output.to(dtype).contiguous()
    E = len(expert_widths)
    xs = _gather_rows(x, gather_map, total_tokens) if gather_map is not None else x.contiguous()
    if activation == "swiglu":
        _check_swiglu_layout(expert_weight_offsets, expert_widths)
        gate = pre_act.to(dtype).contiguous()
        if up_act is None:  # recompute the up projection
            up_act = torch.zeros_like(gate)
            _ops.gemm_up_swiglu(xs, w1.contiguous(), expert_token_offsets, expert_weight_offsets,
                                tokens_per_expert, E, torch.empty_like(gate), up=up_act)
        up = up_act.to(dtype).contiguous()
        grad_act = torch.zeros(total_tokens, 2 * gate.shape[1], device=x.device, dtype=dtype)
        _ops.swiglu_grad(g, gate, up, expert_token_offsets, expert_weight_offsets, E, grad_act)
        _ops.gemm_up_backward(grad_act, xs, w1.contiguous(), expert_token_offsets,
                              expert_weight_offsets, tokens_per_expert, E, grad_x, grad_w1)
        return grad_x, grad_w1
    if activation == "relu_squared":
        grad_act = _ops.relu_squared_grad(g, pre_act)
    else:
        grad_act = g
    _ops.gemm_up_backward(grad_act, xs, w1.contiguous(), expert_token_offsets, expert_weight_offsets,
                          tokens_per_expert, E, grad_x, grad_w1)
    return grad_x, grad_w1


@torch.compiler.disable
def grouped_gemm_down_backward(
    grad_output: torch.Tensor,
    intermediate: torch.Tensor,
    w2: torch.Tensor,
    expert_token_offsets: torch.Tensor,
    expert_weight_offsets: torch.Tensor,
    expert_widths: torch.Tensor,
    tokens_per_expert: torch.Tensor,
    hidden_size: int,
    max_expert_width: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gradients of grouped_gemm_down: (grad_intermediate, grad_w2)."""
    total_tokens = intermediate.shape[0]
    grad_inter = torch.zeros(total_tokens, max_expert_width, device=intermediate.device,
                             dtype=intermediate.dtype)
    grad_w2 = torch.zeros_like(w2)
    if total_tokens == 0:
        return grad_inter, grad_w2
    g = grad_output.to(intermediate.dtype).contiguous()
    E = len(expert_widths)
    _ops.gemm_down_backward(g, intermediate.contiguous(), w2.contiguous(), expert_token_offsets,
                            expert_weight_offsets, tokens_per_expert, E, grad_inter, grad_w2)
    return grad_inter, grad_w2


class GroupedGemmUp(torch.autograd.Function):
    """Autograd function for the grouped up-projection with fused activation.

    With x_flat and gather_map given, backward reads x_flat through gather_map
    instead of keeping the gathered input alive (reference :1440-1460).
    """

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, x, w1, expert_token_offsets, expert_weight_offsets, expert_widths,
                tokens_per_expert, max_expert_width, hidden_size, activation, x_flat, gather_map):
        x = x.to(w1.dtype)
        up_act = None
        if activation == "swiglu":
            # keep the up projection too (the backward needs gate and up)
            _check_activation(activation)
            _check_swiglu_layout(expert_weight_offsets, expert_widths)
            total_tokens = int(expert_token_offsets[-1].item())
            output = torch.zeros(total_tokens, max_expert_width, device=x.device, dtype=x.dtype)
            pre_act = torch.zeros_like(output)
            up_act = torch.zeros_like(output)
            if total_tokens > 0:
                _ops.gemm_up_swiglu(x.contiguous(), w1.contiguous(), expert_token_offsets,
                                    expert_weight_offsets, tokens_per_expert, len(expert_widths),
                                    output, gate=pre_act, up=up_act)
        else:
            output, pre_act = grouped_gemm_up(x, w1, expert_token_offsets, expert_weight_offsets,
                                              expert_widths, tokens_per_expert, max_expert_width,
                                              activation=activation, save_pre_act=True)
        ctx.use_gather_map = x_flat is not None and gather_map is not None
        x_saved = x_flat.to(w1.dtype) if ctx.use_gather_map else x
        ctx.save_for_backward(x_saved, w1, pre_act, expert_token_offsets, expert_weight_offsets,
                              expert_widths, tokens_per_expert,
                              gather_map if ctx.use_gather_map else None, up_act)
        ctx.max_expert_width = max_expert_width
        ctx.hidden_size = hidden_size
        ctx.activation = activation
        return output

    @staticmethod
    @custom_bwd(device_type="cuda")
    @once_differentiable
    def backward(ctx, grad_output):
        (x_for_dw, w1, pre_act, tok_off, w_off, widths, tpe, gather_map,
         up_act) = ctx.saved_tensors
        grad_x, grad_w1 = grouped_gemm_up_backward(
            grad_output, x_for_dw, w1, pre_act, tok_off, w_off, widths, tpe, ctx.hidden_size,
            ctx.activation, gather_map=gather_map, up_act=up_act,
        )
        return grad_x, grad_w1, None, None, None, None, None, None, None, None, None


class GroupedGemmDown(torch.autograd.Function):
    """Autograd function for the grouped down-projection."""

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, intermediate, w2, expert_token_offsets, expert_weight_offsets, expert_widths,
                tokens_per_expert, hidden_size, max_expert_width):
        intermediate = intermediate.to(w2.dtype)
        output = grouped_gemm_down(intermediate, w2, expert_token_offsets, expert_weight_offsets,
                                   expert_widths, tokens_per_expert, hidden_size)
        ctx.save_for_backward(intermediate, w2, expert_token_offsets, expert_weight_offsets,
                              expert_widths, tokens_per_expert)
        ctx.hidden_size = hidden_size
        ctx.max_expert_width = max_expert_width
        return output

    @staticmethod
    @custom_bwd(device_type="cuda")
    @once_differentiable
    def backward(ctx, grad_output):
        intermediate, w2, tok_off, w_off, widths, tpe = ctx.saved_tensors
        grad_inter, grad_w2 = grouped_gemm_down_backward(
            grad_output, intermediate, w2, tok_off, w_off, widths, tpe, ctx.hidden_size,
            ctx.max_expert_width,
        )
        return grad_inter, grad_w2, None, None, None, None, None, None


def grouped_gemm_up_autograd(x, w1, expert_token_offsets, expert_weight_offsets, expert_widths,
                             tokens_per_expert, max_expert_width, hidden_size,
                             activation="relu_squared", x_flat=None, gather_map=None):
    """Grouped up-projection with autograd support."""
    return GroupedGemmUp.apply(x, w1, expert_token_offsets, expert_weight_offsets, expert_widths,
                               tokens_per_expert, max_expert_width, hidden_size, activation,
                               x_flat, gather_map)


def grouped_gemm_down_autograd(intermediate, w2, expert_token_offsets, expert_weight_offsets,
                               expert_widths, tokens_per_expert, hidden_size, max_expert_width):
    """Grouped down-projection with autograd support."""
    return GroupedGemmDown.apply(intermediate, w2, expert_token_offsets, expert_weight_offsets,
                                 expert_widths, tokens_per_expert, hidden_size, max_expert_width)
