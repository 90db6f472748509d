"""CPU oracle for the MoE MLP hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference package triton_moe (hbfreed/
triton-variable-moe), used by the tests, by __graft_entry__.smoke() and by
bench.py's CPU-baseline leg as the checker.  Nothing in the product imports
it.  Each function cites the reference code it restates.

Pinning: the functions are checked against golden vectors produced by the
reference's own Triton kernels run under TRITON_INTERPRET=1 on CPU in fp32
(tests/golden/make_golden.py writes them; tests/test_oracle_golden.py checks
them).

Numerics: GEMMs accumulate in fp32 (numpy float32 matmul).  When `dtype` is
"bf16" the reference's rounding points are applied with round-to-nearest-even
to bfloat16: relu^2 and pre-activation stored in the storage dtype after an
fp32 epilogue (grouped_gemm.py:333-368), the relu^2 derivative computed in
fp32 and cast before the dot (:751-766, :914-928), weighted gather/scatter
products rounded per element and the top-k sum accumulated in fp32
(gather.py:170-174, scatter.py:61-69,133).
"""

from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------- rounding


def round_bf16(a) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(a.shape)


def rounder(dtype: str):
    if dtype in ("bf16", "bfloat16"):
        return round_bf16
    if dtype in ("fp32", "float32"):
        return lambda a: np.asarray(a, dtype=np.float32)
    raise ValueError(dtype)


# ----------------------------------------------------------------- routing


def round_counts(counts: np.ndarray, block_size: int, rounding: str) -> np.ndarray:
    """_cumsum_kernel's rounding modes (fused_cumsum.py:59-66)."""
    c = counts.astype(np.int64)
    if rounding == "up":
        return (c + block_size - 1) // block_size * block_size
    if rounding == "down":
        return c // block_size * block_size
    if rounding == "nearest":
        return (c + block_size // 2) // block_size * block_size
    raise ValueError(rounding)


def fused_route(selected_experts, num_experts: int, block_size: int = 128, rounding: str = "up"):
    """fused_route (fused_cumsum.py:84-171): stable sort, bincount, rounded
    inclusive cumsums, and the keep-mask compaction for "down"/"nearest"."""
    sel = np.asarray(selected_experts).astype(np.int32).reshape(-1)
    order = np.argsort(sel, kind="stable").astype(np.int32)  # torch.sort(stable=True)
    sorted_ids = sel[order]
    tpe = np.bincount(sel, minlength=num_experts).astype(np.int32)
    rounded = round_counts(tpe, block_size, rounding)
    kept = np.minimum(tpe, rounded)
    bins = np.cumsum(kept).astype(np.int32)
    padded_bins = np.cumsum(rounded).astype(np.int32)
    if rounding != "up":  # fused_cumsum.py:154-169
        keep = np.zeros(sel.size, dtype=bool)
        start = 0
        for e in range(num_experts):
            keep[start : start + int(kept[e])] = True
            start += int(tpe[e])
        sorted_ids = sorted_ids[keep]
        order = order[keep]
    return dict(
        bin_ids=sorted_ids.astype(np.int32),
        indices=order.astype(np.int32),
        tokens_per_expert=tpe,
        bins=bins,
        padded_bins=padded_bins,
    )


def _starts(bins, padded_bins):
    b = np.concatenate([[0], np.asarray(bins, np.int64)[:-1]])
    p = np.concatenate([[0], np.asarray(padded_bins, np.int64)[:-1]])
    return b, p


def padded_rows_of(indices, bin_ids, bins, padded_bins) -> np.ndarray:
    """Row of each sorted position in the padded layout (gather.py:35-50)."""
    bstart, pstart = _starts(bins, padded_bins)
    bin_ids = np.asarray(bin_ids, np.int64)
    pos = np.arange(len(bin_ids), dtype=np.int64)
    return pstart[bin_ids] + pos - bstart[bin_ids]


def row_maps(indices, bin_ids, bins, padded_bins, num_assignments: int):
    """(row -> assignment index or -1 for padding, assignment -> row or -1 if dropped)."""
    P = int(padded_bins[-1]) if len(padded_bins) else 0
    r2a = np.full(P, -1, dtype=np.int32)
    a2r = np.full(num_assignments, -1, dtype=np.int32)
    rows = padded_rows_of(indices, bin_ids, bins, padded_bins)
    r2a[rows] = np.asarray(indices, np.int32)
    a2r[np.asarray(indices, np.int64)] = rows.astype(np.int32)
    return r2a, a2r


def precompute_gather_map(indices, bin_ids, bins, padded_bins, top_k: int) -> np.ndarray:
    """precompute_gather_map (grouped_gemm.py:104-149): padding rows map to 0."""
    P = int(padded_bins[-1]) if len(padded_bins) else 0
    gm = np.zeros(P, dtype=np.int32)
    if len(indices):
        rows = padded_rows_of(indices, bin_ids, bins, padded_bins)
        gm[rows] = np.asarray(indices, np.int64) // top_k
    return gm


# ----------------------------------------------------------------- permutation


def padded_gather(x, indices, bin_ids, bins, padded_bins, top_k: int, weights=None, dtype="fp32"):
    """padded_gather (gather.py:13-116) and _weighted_padded_gather (:123-218)."""
    rnd = rounder(dtype)
    x = np.asarray(x, np.float32)
    P = int(padded_bins[-1]) if len(padded_bins) else 0
    out = np.zeros((P, x.shape[1]), np.float32)
    if len(indices):
        rows = padded_rows_of(indices, bin_ids, bins, padded_bins)
        idx = np.asarray(indices, np.int64)
        vals = x[idx // top_k]
        if weights is not None:
            vals = rnd(vals * np.asarray(weights, np.float32)[idx][:, None])
        out[rows] = vals
    return out


def padded_scatter(x, indices, bin_ids, weights, bins, padded_bins, top_k: int, dtype="fp32"):
    """padded_scatter (scatter.py:13-135): per-slot weighted rows, summed over k."""
    rnd = rounder(dtype)
    x = np.asarray(x, np.float32)
    w = np.asarray(weights, np.float32)
    T = w.size // top_k
    inter = np.zeros((T, top_k, x.shape[1]), np.float32)
    if len(indices):
        rows = padded_rows_of(indices, bin_ids, bins, padded_bins)
        idx = np.asarray(indices, np.int64)
        inter[idx // top_k, idx % top_k] = rnd(x[rows] * w[idx][:, None])
    return rnd(inter.sum(axis=1, dtype=np.float32))


# ----------------------------------------------------------------- GEMMs


def _experts(expert_token_offsets, expert_weight_offsets):
    to = np.asarray(expert_token_offsets, np.int64)
    wo = np.asarray(expert_weight_offsets, np.int64)
    for e in range(len(wo) - 1):
        yield e, int(to[e]), int(to[e + 1]), int(wo[e]), int(wo[e + 1])


def grouped_gemm_up(x, w1, expert_token_offsets, expert_weight_offsets, max_expert_width,
                    activation="relu_squared", gather_map=None, dtype="fp32"):
    """grouped_gemm_up (grouped_gemm.py:212-477).  Returns (out, pre_act)."""
    rnd = rounder(dtype)
    x = np.asarray(x, np.float32)
    w1 = np.asarray(w1, np.float32)
    P = int(np.asarray(expert_token_offsets)[-1])
    out = np.zeros((P, max_expert_width), np.float32)
    pre = np.zeros((P, max_expert_width), np.float32)
    for e, r0, r1, c0, c1 in _experts(expert_token_offsets, expert_weight_offsets):
        if r1 == r0:
            continue
        xe = x[np.asarray(gather_map)[r0:r1]] if gather_map is not None else x[r0:r1]
        z = xe @ w1[:, c0:c1]
        if activation == "relu_squared":
            p = np.maximum(z, 0.0)
            pre[r0:r1, : c1 - c0] = rnd(p)
            out[r0:r1, : c1 - c0] = rnd(p * p)
        elif activation == "none":
            out[r0:r1, : c1 - c0] = rnd(z)
        elif activation == "swiglu":
            # grouped_gemm.py:296-358: the expert's columns are gate then up
            # (width w = (c1 - c0) / 2); out = silu(gate) * up, pre_act = gate
            w = (c1 - c0) // 2
            gate, up = z[:, :w], z[:, w:]
            pre[r0:r1, :w] = rnd(gate)
            out[r0:r1, :w] = rnd(gate / (1.0 + np.exp(-gate)) * up)
        else:
            raise NotImplementedError(activation)
    return out, pre


def swiglu_backward(grad_out, gate, up, expert_token_offsets, expert_weight_offsets, dtype="fp32"):
    """The true gradient through out = silu(gate) * up (the reference's own
    swiglu backward is a placeholder, grouped_gemm.py:768-789): returns
    grad_act [P, 2 max_w] with [dgate | dup] in each expert's w1 column layout."""
    rnd = rounder(dtype)
    g = np.asarray(grad_out, np.float32)
    gate = np.asarray(gate, np.float32)
    up = np.asarray(up, np.float32)
    P, maxw = g.shape
    out = np.zeros((P, 2 * maxw), np.float32)
    for e, r0, r1, c0, c1 in _experts(expert_token_offsets, expert_weight_offsets):
        w = (c1 - c0) // 2
        a, u, gg = gate[r0:r1, :w], up[r0:r1, :w], g[r0:r1, :w]
        s = 1.0 / (1.0 + np.exp(-a))
        out[r0:r1, :w] = rnd(gg * u * s * (1.0 + a * (1.0 - s)))
        out[r0:r1, w : 2 * w] = rnd(gg * a * s)
    return out


def grouped_gemm_down(inter, w2, expert_token_offsets, expert_weight_offsets, dtype="fp32"):
    """grouped_gemm_down (grouped_gemm.py:480-651)."""
    rnd = rounder(dtype)
    inter = np.asarray(inter, np.float32)
    w2 = np.asarray(w2, np.float32)
    out = np.zeros((inter.shape[0], w2.shape[1]), np.float32)
    for e, r0, r1, c0, c1 in _experts(expert_token_offsets, expert_weight_offsets):
        if r1 > r0:
            out[r0:r1] = rnd(inter[r0:r1, : c1 - c0] @ w2[c0:c1])
    return out


def relu_squared_grad(grad_out, pre_act, dtype="fp32"):
    """grouped_gemm.py:751-766: where(pre > 0, g * 2 * pre, 0) in fp32, then cast."""
    rnd = rounder(dtype)
    g = np.asarray(grad_out, np.float32)
    p = np.asarray(pre_act, np.float32)
    return rnd(np.where(p > 0, g * 2.0 * p, 0.0).astype(np.float32))


def grouped_gemm_up_backward(grad_output, x, w1, pre_act, expert_token_offsets,
                             expert_weight_offsets, activation="relu_squared", gather_map=None,
                             dtype="fp32"):
    """grouped_gemm_up_backward (grouped_gemm.py:654-967,1165-1290): (grad_x, grad_w1)."""
    rnd = rounder(dtype)
    ga = relu_squared_grad(grad_output, pre_act, dtype) if activation == "relu_squared" \
        else np.asarray(grad_output, np.float32)
    x = np.asarray(x, np.float32)
    w1 = np.asarray(w1, np.float32)
    P = int(np.asarray(expert_token_offsets)[-1])
    gx = np.zeros((P, w1.shape[0]), np.float32)
    gw1 = np.zeros_like(w1)
    for e, r0, r1, c0, c1 in _experts(expert_token_offsets, expert_weight_offsets):
        if r1 == r0:
            continue
        gae = ga[r0:r1, : c1 - c0]
        gx[r0:r1] = rnd(gae @ w1[:, c0:c1].T)
        xe = x[np.asarray(gather_map)[r0:r1]] if gather_map is not None else x[r0:r1]
        gw1[:, c0:c1] = rnd(xe.T @ gae)
    return gx, gw1


def grouped_gemm_down_backward(grad_output, inter, w2, expert_token_offsets,
                               expert_weight_offsets, max_expert_width, dtype="fp32"):
    """grouped_gemm_down_backward (grouped_gemm.py:970-1162,1293-1390): (grad_inter, grad_w2)."""
    rnd = rounder(dtype)
    g = np.asarray(grad_output, np.float32)
    inter = np.asarray(inter, np.float32)
    w2 = np.asarray(w2, np.float32)
    gi = np.zeros((inter.shape[0], max_expert_width), np.float32)
    gw2 = np.zeros_like(w2)
    for e, r0, r1, c0, c1 in _experts(expert_token_offsets, expert_weight_offsets):
        if r1 == r0:
            continue
        gi[r0:r1, : c1 - c0] = rnd(g[r0:r1] @ w2[c0:c1].T)
        gw2[c0:c1] = rnd(inter[r0:r1, : c1 - c0].T @ g[r0:r1])
    return gi, gw2


# ----------------------------------------------------------------- whole layer


def moe_mlp(x_flat, w1, w2, selected_experts, weights, expert_widths, top_k, block_size,
            grad_out=None, dtype="fp32"):
    """TritonMoEMLP.forward after routing (moe.py:185-249) and, when grad_out is
    given, its backward through PaddedScatterOp / GroupedGemmDown /
    GroupedGemmUp / PaddedGatherOp (scatter.py:160-176, grouped_gemm.py:1479-1601,
    gather.py:245-265).  `selected_experts`, `weights` are the flattened top-k
    choice (token-major).  Returns a dict with out (and dx, dw1, dw2)."""
    rnd = rounder(dtype)
    x_flat = rnd(x_flat)
    w1 = rnd(w1)
    w2 = rnd(w2)
    weights = rnd(np.asarray(weights, np.float32).reshape(-1))
    E = len(expert_widths)
    r = fused_route(selected_experts, E, block_size, "up")
    tok_off = np.concatenate([[0], r["padded_bins"]]).astype(np.int64)
    w_off = np.concatenate([[0], np.cumsum(expert_widths)]).astype(np.int64)
    maxw = int(max(expert_widths))
    args = (r["indices"], r["bin_ids"], r["bins"], r["padded_bins"], top_k)
    xg = padded_gather(x_flat, *args, dtype=dtype)
    h, pre = grouped_gemm_up(xg, w1, tok_off, w_off, maxw, "relu_squared", dtype=dtype)
    y = grouped_gemm_down(h, w2, tok_off, w_off, dtype=dtype)
    out = padded_scatter(y, r["indices"], r["bin_ids"], weights, r["bins"], r["padded_bins"],
                         top_k, dtype=dtype)
    res = dict(out=out, routing=r, tok_off=tok_off)
    if grad_out is None:
        return res
    g = rnd(grad_out)
    gy = padded_gather(g, *args, weights=weights, dtype=dtype)
    gi, gw2 = grouped_gemm_down_backward(gy, h, w2, tok_off, w_off, maxw, dtype=dtype)
    gxg, gw1 = grouped_gemm_up_backward(gi, xg, w1, pre, tok_off, w_off, dtype=dtype)
    ones = np.ones(weights.size, np.float32)
    dx = padded_scatter(gxg, r["indices"], r["bin_ids"], ones, r["bins"], r["padded_bins"],
                        top_k, dtype=dtype)
    res.update(dx=dx, dw1=gw1, dw2=gw2)
    return res
