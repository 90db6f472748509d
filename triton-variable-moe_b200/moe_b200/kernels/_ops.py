"""Tensor-level wrappers of the libmoe_b200 C ABI.

These functions take torch tensors, validate them, and launch on the current
CUDA stream.  They never synchronise the host.  Outputs may be passed in
(`out=`) so that callers can reuse or pre-size buffers (the module path sizes
every token-space buffer by an upper bound so that nothing depends on
device-side counts).
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass

import torch

from .._lib import (
    ACT_CODE,
    DTYPE_CODE,
    ROUND_CODE,
    check,
    lib,
    ptr,
    require_cuda,
    stream_handle,
)

_GEMM_DTYPES = (torch.bfloat16, torch.float16, torch.float32)  # fp32 runs on the tf32 MMA

_status_bufs: dict[int, torch.Tensor] = {}

# Number of CUDA kernels launched through this module (host-side count; the
# routing entry point launches one or two).  bench.py reports it per timed region.
launch_count = 0


def _count(n: int = 1) -> None:
    global launch_count
    launch_count += n


_kernel_events: list | None = None
_events_external = False


@contextmanager
def record_kernel_events(external: bool = False):
    """Within the block, every launch of ours is bracketed by CUDA events on its
    launch stream; yields the list of (name, start, end) events.  With
    external=True the events are recorded as event-record nodes when the block
    runs under CUDA-graph capture, so replays of the graph time each kernel."""
    global _kernel_events, _events_external
    prev, _kernel_events = _kernel_events, []
    prev_ext, _events_external = _events_external, external
    try:
        yield _kernel_events
    finally:
        _kernel_events = prev
        _events_external = prev_ext


def _ev_begin():
    if _kernel_events is None:
        return None
    e = torch.cuda.Event(enable_timing=True, external=_events_external)
    e.record()
    return e


def _ev_end(start, name: str) -> None:
    if start is not None:
        e = torch.cuda.Event(enable_timing=True, external=_events_external)
        e.record()
        _kernel_events.append((name, start, e))


def status_buffer(device: torch.device) -> torch.Tensor:
    """Per-device int32 word that kernels set when they detect a device-side
    error (bad expert id, row-capacity overflow, a bounded wait giving up)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _status_bufs.get(idx)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_bufs[idx] = buf
    return buf


def check_device_status(device: torch.device | None = None) -> None:
    """Synchronising check of the device status word; raises and clears it."""
    from .._lib import MoEKernelError, STATUS_TEXT

    device = device or torch.device("cuda", torch.cuda.current_device())
    buf = status_buffer(device)
    v = int(buf.item())
    if v != 0:
        buf.zero_()
        # a launch that gave up may have left its row-block counters non-zero
        reset_up_down_dep_buffer(device)
        raise MoEKernelError(f"device-side error: {STATUS_TEXT.get(v, v)} (status {v})")


def padded_capacity(num_assignments: int, num_experts: int, block_size: int) -> int:
    """Upper bound of the padded row count for any routing outcome."""
    return num_assignments + num_experts * (block_size - 1)


@dataclass
class Routing:
    bin_ids: torch.Tensor  # [A] int32 (first bins[-1] valid)
    indices: torch.Tensor  # [A] int32
    tokens_per_expert: torch.Tensor  # [E] int32
    bins: torch.Tensor  # [E] int32
    padded_bins: torch.Tensor  # [E] int32
    expert_token_offsets: torch.Tensor  # [E+1] int32
    padded_tokens_per_expert: torch.Tensor  # [E] int32
    row_to_assignment: torch.Tensor | None  # [p_capacity] int32
    assignment_to_row: torch.Tensor | None  # [A] int32
    p_capacity: int


def route(
    selected_experts: torch.Tensor,
    num_experts: int,
    block_size: int,
    rounding: str = "up",
    want_rows: bool = True,
) -> Routing:
    require_cuda(selected_experts)
    sel = selected_experts.reshape(-1)
    if sel.dtype not in (torch.int32, torch.int64):
        sel = sel.to(torch.int32)
    sel = sel.contiguous()
    A = sel.numel()
    E = int(num_experts)
    dev = sel.device
    i32 = dict(dtype=torch.int32, device=dev)
    bin_ids = torch.empty(A, **i32)
    indices = torch.empty(A, **i32)
    meta = torch.empty(5 * E + 1, **i32)  # one allocation for the small outputs
    tpe, bins, pbins, ptpe = meta[:E], meta[E : 2 * E], meta[2 * E : 3 * E], meta[3 * E : 4 * E]
    tok_off = meta[4 * E :]
    cap = padded_capacity(A, E, block_size)
    row_asg = torch.empty(max(cap, 1), **i32) if want_rows else None
    asg_row = torch.empty(max(A, 1), **i32) if want_rows else None
    ws_bytes = int(lib.moe_route_workspace_bytes(A, E))
    ws = torch.empty((ws_bytes + 3) // 4, **i32)
    ev = _ev_begin()
    rc = lib.moe_route(
        ptr(sel), 1 if sel.dtype == torch.int64 else 0, A, E, int(block_size), ROUND_CODE[rounding],
        ptr(bin_ids), ptr(indices), ptr(tpe), ptr(bins), ptr(pbins), ptr(tok_off), ptr(ptpe),
        ptr(row_asg), cap, ptr(asg_row), ptr(ws), ws_bytes, ptr(status_buffer(dev)),
        stream_handle(dev),
    )
    _ev_end(ev, "route")
    check(rc, "moe_route")
    _count(1 if A <= 6144 else 2)  # one fused CTA for small problems
    return Routing(bin_ids, indices, tpe, bins, pbins, tok_off, ptpe, row_asg, asg_row, cap)


def router_topk(router_probs: torch.Tensor, top_k: int, normalize: bool, weights_dtype: torch.dtype):
    """(weights [T, k] in weights_dtype, selected [T, k] int32) from fp32 router
    probabilities: torch.topk order, lower index on ties, optional renorm."""
    require_cuda(router_probs)
    p = router_probs.float().contiguous()
    T, E = p.shape
    w = torch.empty(T, top_k, dtype=weights_dtype, device=p.device)
    sel = torch.empty(T, top_k, dtype=torch.int32, device=p.device)
    ev = _ev_begin()
    rc = lib.moe_router_topk(ptr(p), T, E, int(top_k), 1 if normalize else 0, ptr(w),
                             DTYPE_CODE[weights_dtype], ptr(sel), stream_handle(p.device))
    _ev_end(ev, "router_topk")
    check(rc, "moe_router_topk")
    _count(1)
    return w, sel


def router_head(router_logits: torch.Tensor, top_k: int, normalize: bool,
                weights_dtype: torch.dtype, widths_normalized: torch.Tensor,
                lb_coef: torch.Tensor | None = None, ticket: torch.Tensor | None = None):
    """One pass over the router logits: (probs fp32 [T,E], top-k weights [T,k],
    selected int32 [T,k], per-token logsumexp fp32 [T], loss partials).  With
    lb_coef and ticket (a zeroed int32 device word the kernel returns to zero)
    the same launch also forms the auxiliary losses; then (losses fp32 [3],
    f_i [E] in weights_dtype, p_i fp32 [E], z-loss in the logits dtype) follow."""
    require_cuda(router_logits)
    lg = router_logits.contiguous()
    T, E = lg.shape
    dev = lg.device
    probs = torch.empty(T, E, dtype=torch.float32, device=dev)
    w = torch.empty(T, top_k, dtype=weights_dtype, device=dev)
    sel = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    lse = torch.empty(T, dtype=torch.float32, device=dev)
    ws = torch.empty(max(int(lib.moe_router_head_workspace_floats(T, E)), 1), dtype=torch.float32,
                     device=dev)
    wn = widths_normalized.float().contiguous()
    fused = lb_coef is not None and T > 0
    ev = _ev_begin()
    if fused:
        losses = torch.empty(3, dtype=torch.float32, device=dev)
        z = torch.empty((), dtype=lg.dtype, device=dev)
        f_i = torch.empty(E, dtype=weights_dtype, device=dev)
        p_i = torch.empty(E, dtype=torch.float32, device=dev)
        rc = lib.moe_router_head_losses(
            ptr(lg), DTYPE_CODE[lg.dtype], T, E, int(top_k), 1 if normalize else 0, ptr(wn),
            ptr(probs), ptr(w), DTYPE_CODE[weights_dtype], ptr(sel), ptr(lse), ptr(ws),
            ptr(lb_coef.float().contiguous()), ptr(losses), ptr(f_i), ptr(p_i), ptr(z),
            ptr(ticket), stream_handle(dev))
        name = "moe_router_head_losses"
    else:
        rc = lib.moe_router_head(ptr(lg), DTYPE_CODE[lg.dtype], T, E, int(top_k),
                                 1 if normalize else 0, ptr(wn), ptr(probs), ptr(w),
                                 DTYPE_CODE[weights_dtype], ptr(sel), ptr(lse), ptr(ws),
                                 stream_handle(dev))
        name = "moe_router_head"
    _ev_end(ev, "router_head")
    check(rc, name)
    _count(1)
    if fused:
        return probs, w, sel, lse, ws, (losses, f_i, p_i, z)
    return probs, w, sel, lse, ws


def aux_losses(ws: torch.Tensor, num_tokens: int, tokens_per_expert: torch.Tensor | None,
               lb_coef: torch.Tensor, logits_dtype: torch.dtype, f_dtype: torch.dtype,
               out: tuple | None = None):
    """(losses fp32 [3] = z, load balance, compute; f_i [E]; p_i fp32 [E];
    z-loss in the logits dtype).  tokens_per_expert None: the router head's own
    selection counts in ws are used.  out: preallocated (losses, f_i, p_i, z)."""
    dev = ws.device
    E = lb_coef.numel()
    if out is None:
        out = (torch.empty(3, dtype=torch.float32, device=dev), torch.empty(E, dtype=f_dtype, device=dev),
               torch.empty(E, dtype=torch.float32, device=dev),
               torch.empty((), dtype=logits_dtype, device=dev))
    losses, f_i, p_i, z = out
    tpe = _meta(tokens_per_expert) if tokens_per_expert is not None else None
    ev = _ev_begin()
    rc = lib.moe_aux_losses(ptr(ws), int(num_tokens), E, ptr(tpe),
                            ptr(lb_coef.float().contiguous()), DTYPE_CODE[logits_dtype],
                            ptr(losses), ptr(f_i), DTYPE_CODE[f_dtype], ptr(p_i), ptr(z),
                            stream_handle(dev))
    _ev_end(ev, "aux_losses")
    check(rc, "moe_aux_losses")
    _count(1)
    return losses, f_i, p_i, z


def build_row_map(
    indices: torch.Tensor,
    bin_ids: torch.Tensor,
    bins: torch.Tensor,
    padded_bins: torch.Tensor,
    padded_rows: int,
    num_assignments: int,
    want_row_to_assignment: bool = True,
    want_assignment_to_row: bool = True,
) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    require_cuda(indices, bin_ids, bins, padded_bins)
    dev = indices.device
    ind = indices.to(torch.int32).contiguous()
    bid = bin_ids.to(torch.int32).contiguous()
    b = bins.to(torch.int32).contiguous()
    pb = padded_bins.to(torch.int32).contiguous()
    r2a = torch.empty(max(padded_rows, 1), dtype=torch.int32, device=dev) if want_row_to_assignment else None
    a2r = torch.empty(max(num_assignments, 1), dtype=torch.int32, device=dev) if want_assignment_to_row else None
    rc = lib.moe_build_row_map(
        ptr(ind), ptr(bid), ptr(b), ptr(pb), ind.numel(), padded_rows, ptr(r2a),
        num_assignments, ptr(a2r), ptr(status_buffer(dev)), stream_handle(dev),
    )
    check(rc, "moe_build_row_map")
    _count(1)
    return r2a, a2r


def gather_map(row_to_assignment: torch.Tensor, padded_rows: int, top_k: int) -> torch.Tensor:
    dev = row_to_assignment.device
    out = torch.empty(padded_rows, dtype=torch.int32, device=dev)
    check(lib.moe_gather_map(ptr(row_to_assignment), padded_rows, top_k, ptr(out), stream_handle(dev)),
          "moe_gather_map")
    _count()
    return out


def gather(
    x: torch.Tensor,
    row_map: torch.Tensor,
    map_div: int,
    rows: int,
    out: torch.Tensor | None = None,
    rows_device: torch.Tensor | None = None,
    weights: torch.Tensor | None = None,
) -> torch.Tensor:
    """out[r] = x[row_map[r] // map_div] (* weights[row_map[r]]), zero where row_map < 0."""
    require_cuda(x, row_map)
    if x.stride(-1) != 1:
        x = x.contiguous()
    H = x.shape[1]
    if out is None:
        out = torch.empty(rows, H, dtype=x.dtype, device=x.device)
    if weights is not None:
        weights = weights.to(x.dtype).contiguous()
    ev = _ev_begin()
    rc = lib.moe_padded_gather(
        ptr(x), x.stride(0), H, ptr(row_map), int(map_div), int(rows), ptr(rows_device),
        ptr(weights), ptr(out), out.stride(0), DTYPE_CODE[x.dtype], stream_handle(x.device),
    )
    _ev_end(ev, "gather" if weights is None else "weighted_gather")
    check(rc, "moe_padded_gather")
    _count(1)
    return out


def combine(
    y: torch.Tensor,
    assignment_to_row: torch.Tensor,
    num_tokens: int,
    top_k: int,
    weights: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """out[t] = sum_j round(y[row(t, j)] * w[t*k+j]) (unit weights when None)."""
    require_cuda(y, assignment_to_row)
    if y.stride(-1) != 1:
        y = y.contiguous()
    H = y.shape[1]
    if out is None:
        out = torch.empty(num_tokens, H, dtype=y.dtype, device=y.device)
    if weights is not None:
        weights = weights.to(y.dtype).contiguous()
    ev = _ev_begin()
    rc = lib.moe_padded_scatter(
        ptr(y), y.stride(0), H, ptr(assignment_to_row), int(num_tokens), int(top_k),
        ptr(weights), ptr(out), out.stride(0), DTYPE_CODE[y.dtype], stream_handle(y.device),
    )
    _ev_end(ev, "combine")
    check(rc, "moe_padded_scatter")
    _count(1)
    return out


def relu_squared_grad(grad_out: torch.Tensor, pre_act: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    require_cuda(grad_out, pre_act)
    g = grad_out.contiguous()
    p = pre_act.to(g.dtype).contiguous()
    if out is None:
        out = torch.empty_like(g)
    rc = lib.moe_relu_squared_grad(ptr(g), ptr(p), g.shape[0], g.shape[1], g.stride(0), ptr(out),
                                   DTYPE_CODE[g.dtype], stream_handle(g.device))
    check(rc, "moe_relu_squared_grad")
    _count(1)
    return out


def _gemm_check(*ts: torch.Tensor) -> None:
    require_cuda(*ts)
    dt = ts[0].dtype
    for t in ts:
        if t.dtype != dt:
            raise TypeError(f"grouped GEMM operands must share a dtype, got {dt} and {t.dtype}")
        if t.stride(-1) != 1:
            raise ValueError("grouped GEMM operands must be row-major contiguous in the last dim")
    if dt not in _GEMM_DTYPES:
        raise NotImplementedError(
            f"grouped GEMM dtype {dt}: the sm_100a kernels take bf16/fp16 (kind::f16) or fp32 (kind::tf32) operands with fp32 accumulation"
        )


def _meta(t: torch.Tensor | None) -> torch.Tensor | None:
    if t is None:
        return None
    return t if (t.dtype == torch.int32 and t.is_contiguous()) else t.to(torch.int32).contiguous()


def gemm_up(x, w1, tok_off, w_off, tok_cnt, num_experts, activation, out, pre_act=None, tile_n=0):
    _gemm_check(x, w1, out)
    tok_off, w_off, tok_cnt = _meta(tok_off), _meta(w_off), _meta(tok_cnt)
    H, TW = w1.shape
    ev = _ev_begin()
    rc = lib.moe_grouped_gemm_up(
        ptr(x), x.shape[0], x.stride(0), ptr(w1), H, TW, ptr(tok_off), ptr(w_off), ptr(tok_cnt),
        int(num_experts), ACT_CODE[activation], ptr(out), ptr(pre_act), out.stride(0),
        DTYPE_CODE[x.dtype], int(tile_n), ptr(status_buffer(x.device)), stream_handle(x.device),
    )
    _ev_end(ev, "grouped_gemm_up")
    check(rc, "moe_grouped_gemm_up")
    _count(1)
    return out


def gemm_up_swiglu(x, w1, tok_off, w_off, tok_cnt, num_experts, out, gate=None, up=None,
                   tile_n=0):
    """out = silu(x @ gate_e) * (x @ up_e) per expert (w1 columns: gate block then
    up block per expert, w_off stepping by 2 w_e); gate / up optionally stored."""
    _gemm_check(x, w1, out)
    for t in (gate, up):
        if t is not None and (t.stride(0) != out.stride(0) or t.dtype != out.dtype):
            raise ValueError("gate / up must match out's dtype and row stride")
    tok_off, w_off, tok_cnt = _meta(tok_off), _meta(w_off), _meta(tok_cnt)
    H, TW = w1.shape
    ev = _ev_begin()
    rc = lib.moe_grouped_gemm_up_swiglu(
        ptr(x), x.shape[0], x.stride(0), ptr(w1), H, TW, ptr(tok_off), ptr(w_off), ptr(tok_cnt),
        int(num_experts), ptr(out), ptr(gate), ptr(up), out.stride(0), DTYPE_CODE[x.dtype],
        int(tile_n), ptr(status_buffer(x.device)), stream_handle(x.device),
    )
    _ev_end(ev, "grouped_gemm_up")
    check(rc, "moe_grouped_gemm_up_swiglu")
    _count(1)
    return out


def swiglu_grad(grad_out, gate, up, tok_off, w_off, num_experts, out):
    """[dgate | dup] per expert in w1's gate/up column layout (out: [rows, >= 2 max_w])."""
    require_cuda(grad_out, gate, up, out)
    if not (grad_out.stride(0) == gate.stride(0) == up.stride(0)):
        raise ValueError("grad_out, gate and up must share a row stride")
    rc = lib.moe_swiglu_grad(ptr(grad_out), ptr(gate), ptr(up), grad_out.shape[0],
                             grad_out.stride(0), ptr(_meta(tok_off)), ptr(_meta(w_off)),
                             int(num_experts), ptr(out), out.stride(0),
                             DTYPE_CODE[grad_out.dtype], stream_handle(grad_out.device))
    check(rc, "moe_swiglu_grad")
    _count(1)
    return out


_dep_buffers: dict = {}
# replaced (smaller) counter buffers stay allocated: a CUDA graph captured with
# one keeps its address
_dep_buffers_retired: list = []


def up_down_dep_buffer(device: torch.device, rows: int, num_experts: int) -> torch.Tensor:
    """Zeroed int32 row-block counters for gemm_up_down (every launch returns
    them to zero); one per device, grown on demand.  gemm_up_down launches on
    one device never overlap: see _order_up_down."""
    words = int(lib.moe_up_down_dep_words(rows, num_experts))
    device = torch.device(device)
    buf = _dep_buffers.get(device)
    if buf is None or buf.numel() < words:
        if torch.cuda.is_current_stream_capturing():
            # a zero fill recorded into a graph runs only at replay
            raise RuntimeError(
                "gemm_up_down: run the layer once eagerly at this size before capturing "
                "it in a CUDA graph (its counter buffer is allocated on first use)")
        if buf is not None:
            _dep_buffers_retired.append(buf)
        buf = torch.zeros(max(words, 1), dtype=torch.int32, device=device)
        _dep_buffers[device] = buf
    return buf


def reset_up_down_dep_buffer(device: torch.device) -> None:
    """Zero the device's gemm_up_down counters (stream-ordered).  Every launch
    that completes normally leaves them at zero; one that gave up (a device
    wait ran out, status MOE_ERR_TIMEOUT) may not, and a later launch could
    then pass its waits too early."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _dep_buffers.get(torch.device("cuda", idx))
    if buf is not None:
        buf.zero_()


_up_down_last_stream: dict = {}


def _order_up_down(device: torch.device) -> None:
    """Order this gemm_up_down launch after the device's previous one when that
    ran on another stream.  The fused launch's down tiles wait for other CTAs'
    up tiles, so its whole grid must be resident; two such grids overlapping on
    unordered streams could hold SMs against each other (their waits would run
    out, MOE_ERR_TIMEOUT), and they share the row-block counters.  One stream:
    nothing is added.  While capturing a CUDA graph the capture's own ordering
    applies (a wait on work outside the capture is not allowed)."""
    if torch.cuda.is_current_stream_capturing():
        return
    idx = device.index if device.index is not None else torch.cuda.current_device()
    cur = torch.cuda.current_stream(torch.device("cuda", idx))
    prev = _up_down_last_stream.get(idx)
    if prev is not None and prev.cuda_stream != cur.cuda_stream:
        cur.wait_stream(prev)
    _up_down_last_stream[idx] = cur


def gemm_up_down(x, w1, w2, tok_off, w_off, tok_cnt, num_experts, inter, pre_act, out,
                 tile_n_width=0, tile_n_hidden=0):
    """inter = relu(x @ w1_e)^2 (pre_act = relu(x @ w1_e)), out = inter @ w2_e in
    one launch; down tiles start as their row blocks of inter are complete."""
    _gemm_check(x, w1, w2, inter, out)
    tok_off, w_off, tok_cnt = _meta(tok_off), _meta(w_off), _meta(tok_cnt)
    H, TW = w1.shape
    dep = up_down_dep_buffer(x.device, x.shape[0], num_experts)
    _order_up_down(x.device)
    ev = _ev_begin()
    rc = lib.moe_grouped_gemm_up_down(
        ptr(x), x.shape[0], x.stride(0), ptr(w1), ptr(w2), H, TW, ptr(tok_off), ptr(w_off),
        ptr(tok_cnt), int(num_experts), ptr(inter), ptr(pre_act), inter.stride(0), ptr(out),
        out.stride(0), ptr(dep), dep.numel(), DTYPE_CODE[x.dtype], int(tile_n_width),
        int(tile_n_hidden), ptr(status_buffer(x.device)), stream_handle(x.device),
    )
    _ev_end(ev, "grouped_gemm_up_down")
    if rc != 0:
        reset_up_down_dep_buffer(x.device)
    check(rc, "moe_grouped_gemm_up_down")
    _count(1)
    return out


def gemm_down(inter, w2, tok_off, w_off, tok_cnt, num_experts, out, tile_n=0):
    _gemm_check(inter, w2, out)
    tok_off, w_off, tok_cnt = _meta(tok_off), _meta(w_off), _meta(tok_cnt)
    TW, H = w2.shape
    ev = _ev_begin()
    rc = lib.moe_grouped_gemm_down(
        ptr(inter), inter.shape[0], inter.stride(0), ptr(w2), H, TW, ptr(tok_off), ptr(w_off),
        ptr(tok_cnt), int(num_experts), ptr(out), out.stride(0), DTYPE_CODE[inter.dtype],
        int(tile_n), ptr(status_buffer(inter.device)), stream_handle(inter.device),
    )
    _ev_end(ev, "grouped_gemm_down")
    check(rc, "moe_grouped_gemm_down")
    _count(1)
    return out


def gemm_up_dx(grad_act, w1, tok_off, w_off, tok_cnt, num_experts, out, tile_n=0):
    _gemm_check(grad_act, w1, out)
    tok_off, w_off, tok_cnt = _meta(tok_off), _meta(w_off), _meta(tok_cnt)
    H, TW = w1.shape
    ev = _ev_begin()
    rc = lib.moe_grouped_gemm_up_dx(
        ptr(grad_act), grad_act.shape[0], grad_act.stride(0), ptr(w1), H, TW, ptr(tok_off),
        ptr(w_off), ptr(tok_cnt), int(num_experts), ptr(out), out.stride(0),
        DTYPE_CODE[grad_act.dtype], int(tile_n), ptr(status_buffer(w1.device)),
        stream_handle(w1.device),
    )
    _ev_end(ev, "grouped_gemm_up_dx")
    check(rc, "moe_grouped_gemm_up_dx")
    _count(1)
    return out


def gemm_up_dw(x, grad_act, tok_off, w_off, num_experts, out, tile_n=0):
    _gemm_check(x, grad_act, out)
    tok_off, w_off = _meta(tok_off), _meta(w_off)
    H, TW = out.shape
    ev = _ev_begin()
    rc = lib.moe_grouped_gemm_up_dw(
        ptr(x), x.shape[0], x.stride(0), ptr(grad_act), grad_act.stride(0), H, TW, ptr(tok_off),
        ptr(w_off), int(num_experts), ptr(out), DTYPE_CODE[x.dtype], int(tile_n),
        ptr(status_buffer(x.device)), stream_handle(x.device),
    )
    _ev_end(ev, "grouped_gemm_up_dw")
    check(rc, "moe_grouped_gemm_up_dw")
    _count(1)
    return out


def gemm_down_dinter(grad_y, w2, tok_off, w_off, tok_cnt, num_experts, out, pre_act=None, tile_n=0):
    _gemm_check(grad_y, w2, out)
    tok_off, w_off, tok_cnt = _meta(tok_off), _meta(w_off), _meta(tok_cnt)
    TW, H = w2.shape
    ld_pre = pre_act.stride(0) if pre_act is not None else 0
    ev = _ev_begin()
    rc = lib.moe_grouped_gemm_down_dinter(
        ptr(grad_y), grad_y.shape[0], grad_y.stride(0), ptr(w2), H, TW, ptr(tok_off), ptr(w_off),
        ptr(tok_cnt), int(num_experts), ptr(pre_act), ld_pre, ptr(out), out.stride(0),
        DTYPE_CODE[grad_y.dtype], int(tile_n), ptr(status_buffer(w2.device)),
        stream_handle(w2.device),
    )
    _ev_end(ev, "grouped_gemm_down_dinter")
    check(rc, "moe_grouped_gemm_down_dinter")
    _count(1)
    return out


def gemm_down_dw(inter, grad_y, tok_off, w_off, num_experts, out, tile_n=0):
    _gemm_check(inter, grad_y, out)
    tok_off, w_off = _meta(tok_off), _meta(w_off)
    TW, H = out.shape
    ev = _ev_begin()
    rc = lib.moe_grouped_gemm_down_dw(
        ptr(inter), inter.shape[0], inter.stride(0), ptr(grad_y), grad_y.stride(0), H, TW,
        ptr(tok_off), ptr(w_off), int(num_experts), ptr(out), DTYPE_CODE[inter.dtype], int(tile_n),
        ptr(status_buffer(inter.device)), stream_handle(inter.device),
    )
    _ev_end(ev, "grouped_gemm_down_dw")
    check(rc, "moe_grouped_gemm_down_dw")
    _count(1)
    return out


def gemm_down_backward(grad_y, inter, w2, tok_off, w_off, tok_cnt, num_experts, grad_inter, grad_w2,
                       pre_act=None, tile_n_width=0, tile_n_hidden=0):
    """dIntermediate (relu^2 derivative fused when pre_act is given) and dW2 in one launch."""
    _gemm_check(grad_y, inter, w2, grad_inter, grad_w2)
    tok_off, w_off, tok_cnt = _meta(tok_off), _meta(w_off), _meta(tok_cnt)
    TW, H = w2.shape
    ld_pre = pre_act.stride(0) if pre_act is not None else 0
    ev = _ev_begin()
    rc = lib.moe_grouped_gemm_down_backward(
        ptr(grad_y), grad_y.shape[0], grad_y.stride(0), ptr(inter), inter.stride(0), ptr(w2), H,
        TW, ptr(tok_off), ptr(w_off), ptr(tok_cnt), int(num_experts), ptr(pre_act), ld_pre,
        ptr(grad_inter), grad_inter.stride(0), ptr(grad_w2), DTYPE_CODE[grad_y.dtype],
        int(tile_n_width), int(tile_n_hidden), ptr(status_buffer(w2.device)),
        stream_handle(w2.device),
    )
    _ev_end(ev, "grouped_gemm_down_backward")
    check(rc, "moe_grouped_gemm_down_backward")
    _count(1)


def gemm_up_backward(grad_act, x, w1, tok_off, w_off, tok_cnt, num_experts, grad_x, grad_w1,
                     tile_n_width=0, tile_n_hidden=0):
    """dX and dW1 from the activation gradient in one launch (grad_x may be None:
    dW1 only)."""
    if grad_x is None:
        return gemm_up_dw(x, grad_act, tok_off, w_off, num_experts, grad_w1, tile_n=tile_n_width)
    _gemm_check(grad_act, x, w1, grad_x, grad_w1)
    tok_off, w_off, tok_cnt = _meta(tok_off), _meta(w_off), _meta(tok_cnt)
    H, TW = w1.shape
    ev = _ev_begin()
    rc = lib.moe_grouped_gemm_up_backward(
        ptr(grad_act), grad_act.shape[0], grad_act.stride(0), ptr(x), x.stride(0), ptr(w1), H, TW,
        ptr(tok_off), ptr(w_off), ptr(tok_cnt), int(num_experts), ptr(grad_x), grad_x.stride(0),
        ptr(grad_w1), DTYPE_CODE[grad_act.dtype], int(tile_n_width), int(tile_n_hidden),
        ptr(status_buffer(w1.device)), stream_handle(w1.device),
    )
    _ev_end(ev, "grouped_gemm_up_backward")
    check(rc, "moe_grouped_gemm_up_backward")
    _count(1)
