"""Mixture-of-experts MLP layer on the sm_100a kernels of this package.

Drop-in for triton_moe/moe.py: `TritonMoEConfig` (:30-39) and `TritonMoEMLP`
(:42-518) keep their names, constructor, parameters (`router.weight`, `w1`,
`w2`: identical state_dict keys and layouts), buffers, `forward`,
`forward_with_intermediates` and `forward_profiled`.

The training path differs from the reference in how it is executed, not in
what it computes:
  * the layer body after routing (route -> gather -> up(relu^2) -> down ->
    combine, and the mirrored backward) is one autograd Function that calls
    the C-ABI kernels directly;
  * every token-space buffer is sized by the worst-case padded row count
    (assignments + experts * (block_size - 1)), and every kernel reads the
    actual per-expert extents from device memory, so the forward and the
    backward never synchronise with the host and can be captured in a CUDA
    graph;
  * the relu^2 derivative is fused into the epilogue of the down-projection's
    dIntermediate GEMM, and the unit-weight scatter of the gather backward is
    the same single-pass combine kernel as the forward scatter.
Numerics follow the reference's rounding points (fp32 accumulation, relu^2
applied in fp32 before the store, derivative computed in fp32 and rounded
before the dX / dW GEMMs).  As in the reference, the routing weights receive
no gradient from the layer output (scatter.py:160-176).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd.function import once_differentiable

from .kernels import (
    _ops,
    fused_route,
    grouped_gemm_down,
    grouped_gemm_up,
    padded_gather,
    padded_scatter,
)


@dataclass
class TritonMoEConfig:
    """Configuration of the MoE layer (same fields as triton_moe.TritonMoEConfig)."""

    n_embd: int = 768
    expert_sizes: list = field(default_factory=lambda: [(64, 256)])
    num_active_experts: int = 8
    norm_topk_prob: bool = True
    block_size: int = 64
    use_megablocks_gather_scatter: bool = False


@dataclass
class _Plan:
    """Static per-layer launch plan (host constants + device offset table)."""

    num_experts: int
    top_k: int
    block_size: int
    hidden: int
    max_width: int
    w_off: torch.Tensor  # [E+1] int32, device
    tile_n_width: int  # N tile for GEMMs whose N is an expert width
    tile_n_hidden: int  # N tile for GEMMs whose N is the hidden size


class _MoEMLPFunction(torch.autograd.Function):
    """route -> gather -> up(relu^2) -> down -> combine, and the backward."""

    @staticmethod
    def forward(ctx, x_flat, w1, w2, weights, selected, plan: _Plan):
        ctx.set_materialize_grads(False)  # no zero-filled grads for unused outputs
        T, H = x_flat.shape
        E, k = plan.num_experts, plan.top_k
        r = _ops.route(selected, E, plan.block_size, "up")
        cap = r.p_capacity
        rows = max(cap, 1)
        p_dev = r.expert_token_offsets[E:]  # device scalar: padded row count
        dev, dt = x_flat.device, x_flat.dtype
        train = any(ctx.needs_input_grad[:3])

        xg = torch.empty(rows, H, device=dev, dtype=dt)
        _ops.gather(x_flat, r.row_to_assignment, k, cap, out=xg, rows_device=p_dev)
        h = torch.empty(rows, plan.max_width, device=dev, dtype=dt)
        pre = torch.empty_like(h) if train else None
        # up (relu^2) and down in one launch: down tiles start as soon as their
        # rows of h are complete
        y = torch.empty(rows, H, device=dev, dtype=dt)
        _ops.gemm_up_down(xg, w1, w2, r.expert_token_offsets, plan.w_off, None, E, h, pre, y,
                          tile_n_width=plan.tile_n_width, tile_n_hidden=plan.tile_n_hidden)
        out = _ops.combine(y, r.assignment_to_row, T, k, weights=weights)

        if train:
            ctx.save_for_backward(xg, h, pre, weights, w1, w2, r.row_to_assignment,
                                  r.assignment_to_row, r.expert_token_offsets)
            ctx.plan = plan
            ctx.cap = cap
            ctx.T = T
        ctx.mark_non_differentiable(r.tokens_per_expert)
        return out, r.tokens_per_expert

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out, _grad_tpe):
        if grad_out is None:
            return None, None, None, None, None, None
        xg, h, pre, weights, w1, w2, r2a, a2r, tok_off = ctx.saved_tensors
        plan = ctx.plan
        E, k, cap = plan.num_experts, plan.top_k, ctx.cap
        rows = max(cap, 1)
        p_dev = tok_off[E:]
        dev, dt = xg.device, xg.dtype
        H = xg.shape[1]
        grad_out = grad_out.to(dt)

        # scatter backward: weighted gather of the output gradient
        gy = torch.empty(rows, H, device=dev, dtype=dt)
        _ops.gather(grad_out, r2a, k, cap, out=gy, rows_device=p_dev, weights=weights)
        # down backward: dIntermediate with the relu^2 derivative fused, and dW2,
        # in one launch
        dact = torch.empty(rows, plan.max_width, device=dev, dtype=dt)
        gw2 = torch.empty_like(w2)
        _ops.gemm_down_backward(gy, h, w2, tok_off, plan.w_off, None, E, dact, gw2, pre_act=pre,
                                tile_n_width=plan.tile_n_width, tile_n_hidden=plan.tile_n_hidden)
        # up backward: dX (gathered space) and dW1 in one launch
        gxg = torch.empty(rows, H, device=dev, dtype=dt) if ctx.needs_input_grad[0] else None
        gw1 = torch.empty_like(w1)
        _ops.gemm_up_backward(dact, xg, w1, tok_off, plan.w_off, None, E, gxg, gw1,
                              tile_n_width=plan.tile_n_width, tile_n_hidden=plan.tile_n_hidden)
        # gather backward: unit-weight combine of the k copies of each token
        gx = _ops.combine(gxg, a2r, ctx.T, k, weights=None) if gxg is not None else None
        if not ctx.needs_input_grad[1]:
            gw1 = None
        if not ctx.needs_input_grad[2]:
            gw2 = None
        return gx, gw1, gw2, None, None, None


class _RouterHead(torch.autograd.Function):
    """sigmoid + top-k + renorm + per-token logsumexp of the router logits (one
    kernel), then the auxiliary losses from its partial sums and selection
    counts (a second one-block kernel, on `aux_stream` when given so that it
    overlaps the routing and expert GEMMs; the caller joins that stream before
    the loss values are used).  Differentiable output: the fp32 probabilities
    (d sigmoid = p(1-p)); the loss values are handed to _AuxLosses, which
    carries their gradients."""

    @staticmethod
    def forward(ctx, logits, top_k, normalize, weights_dtype, widths_normalized, lb_coef,
                aux_stream):
        ctx.set_materialize_grads(False)  # no zero-filled grads for unused outputs
        probs, w, sel, lse, ws = _ops.router_head(logits, top_k, normalize, weights_dtype,
                                                  widths_normalized)
        T, E = logits.shape
        dev = logits.device
        out = (torch.empty(3, dtype=torch.float32, device=dev),
               torch.empty(E, dtype=weights_dtype, device=dev),
               torch.empty(E, dtype=torch.float32, device=dev),
               torch.empty((), dtype=logits.dtype, device=dev))
        if aux_stream is None:
            _ops.aux_losses(ws, T, None, lb_coef, logits.dtype, weights_dtype, out=out)
        else:
            aux_stream.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(aux_stream):
                _ops.aux_losses(ws, T, None, lb_coef, logits.dtype, weights_dtype, out=out)
            ws.record_stream(aux_stream)
        losses, f_i, _p_i, z = out
        ctx.save_for_backward(probs)
        ctx.logits_dtype = logits.dtype
        ctx.mark_non_differentiable(w, sel, lse, losses, f_i, z)
        return probs, w, sel, lse, losses, f_i, z

    @staticmethod
    @once_differentiable
    def backward(ctx, g_probs, _w, _sel, _lse, _losses, _f_i, _z):
        (probs,) = ctx.saved_tensors
        g = None
        if g_probs is not None:
            g = (g_probs * probs * (1.0 - probs)).to(ctx.logits_dtype)
        return g, None, None, None, None, None, None


class _AuxLosses(torch.autograd.Function):
    """router_z_loss, load_balance_loss, compute_loss and f_i as the router head
    computed them (forward passes them through).  Backward restates the
    gradients of the reference's torch expressions (moe.py:253-303)."""

    @staticmethod
    def forward(ctx, logits, probs, lse, losses, f_i, z, lb_coef, widths_normalized):
        ctx.set_materialize_grads(False)  # no zero-filled grads for unused outputs
        lb = losses[1]
        cl = losses[2]
        ctx.save_for_backward(logits, lse, f_i, lb_coef, widths_normalized)
        ctx.mark_non_differentiable(f_i)
        return z, lb, cl, f_i

    @staticmethod
    @once_differentiable
    def backward(ctx, g_z, g_lb, g_cl, _g_f):
        logits, lse, f_i, lb_coef, wn = ctx.saved_tensors
        T, E = logits.shape
        g_logits = g_probs = None
        if g_z is not None:
            # d/dlogits mean_t lse_t^2 = (2 lse_t / T) softmax(logits_t)
            coef = g_z.float() * 2.0 * lse / T
            g_logits = (torch.softmax(logits.float(), dim=-1) * coef[:, None]).to(logits.dtype)
        if g_lb is not None or g_cl is not None:
            gp = torch.zeros(E, dtype=torch.float32, device=logits.device)
            if g_cl is not None:
                gp = gp + g_cl.float() * wn.float()
            if g_lb is not None:
                gp = gp + g_lb.float() * lb_coef.float() * f_i.float()
            g_probs = (gp / T).expand(T, E)
        return g_logits, g_probs, None, None, None, None, None, None


class TritonMoEMLP(nn.Module):
    """Mixture-of-experts MLP with variable-width experts (drop-in for
    triton_moe.TritonMoEMLP)."""

    def __init__(self, config: TritonMoEConfig):
        super().__init__()
        self.config = config
        self.num_experts = sum(count for count, _ in config.expert_sizes)
        self.num_active_experts = config.num_active_experts
        self.norm_topk_prob = config.norm_topk_prob
        self.block_size = config.block_size

        self.expert_widths = []
        self.expert_offsets = [0]
        for count, size in config.expert_sizes:
            assert size % self.block_size == 0, (
                f"expert sizes must be divisible by {self.block_size}"
            )
            for _ in range(count):
                self.expert_widths.append(size)
                self.expert_offsets.append(self.expert_offsets[-1] + size)
        self.total_expert_width = self.expert_offsets[-1]
        self.max_expert_width = max(self.expert_widths)

        self.router = nn.Linear(config.n_embd, self.num_experts, bias=False)
        self.w1 = nn.Parameter(torch.empty(config.n_embd, self.total_expert_width))
        self.w2 = nn.Parameter(torch.empty(self.total_expert_width, config.n_embd))
        nn.init.trunc_normal_(self.w1, mean=0.0, std=0.02, a=-0.06, b=0.06)
        nn.init.trunc_normal_(self.w2, mean=0.0, std=0.02, a=-0.06, b=0.06)

        self.register_buffer("expert_widths_t", torch.tensor(self.expert_widths, dtype=torch.int32),
                             persistent=False)
        self.register_buffer("expert_weight_offsets_t",
                             torch.tensor(self.expert_offsets, dtype=torch.int32), persistent=False)

        mean_w = sum(self.expert_widths) / self.num_experts
        self.register_buffer(
            "expert_widths_normalized",
            torch.tensor([w / mean_w for w in self.expert_widths], dtype=torch.float32),
            persistent=False,
        )

        # experts of a (count > 1) size class form a load-balance group; singleton
        # classes are left out of the grouped loss (moe.py:108-146)
        expert_to_group, group_sizes, gidx = [], [], 0
        for count, _size in config.expert_sizes:
            expert_to_group += [gidx if count > 1 else -1] * count
            if count > 1:
                group_sizes.append(count)
                gidx += 1
        num_groups = len(group_sizes)
        # load_balance_loss = sum_e lb_coef[e] * f_i[e] * p_i[e]: the three cases of
        # moe.py:276-303 (uniform widths, no size group with >1 expert, groups)
        if len(set(self.expert_widths)) == 1:
            coef = [float(self.num_experts)] * self.num_experts
        elif num_groups == 0:
            coef = [1.0] * self.num_experts
        else:
            coef = [
                (group_sizes[g] / num_groups) if g >= 0 else 0.0
                for g in expert_to_group
            ]
        # kept out of the module's buffers so that module.to(dtype) does not round it
        self._lb_coef_values = coef
        self._plan_cache: _Plan | None = None

    # ------------------------------------------------------------------ helpers
    def _plan(self) -> _Plan:
        p = self._plan_cache
        w_off = self.expert_weight_offsets_t
        if p is None or p.w_off is not w_off:
            # N tile 256 once any expert is wider than 128 (narrower experts then
            # leave part of a tile idle, which measured cheaper than twice the tiles)
            tn_w = 256 if self.max_expert_width > 128 else 128
            tn_h = 256 if self.config.n_embd % 256 == 0 else 128
            p = _Plan(self.num_experts, self.num_active_experts, self.block_size,
                      self.config.n_embd, self.max_expert_width, w_off, tn_w, tn_h)
            self._plan_cache = p
        return p

    def _fp32(self, name: str) -> torch.Tensor:
        """fp32 view of a float buffer (the module may have been cast to bf16, which
        rounds the buffer like the reference's); cached per buffer version."""
        buf = getattr(self, name)
        if buf.dtype == torch.float32:
            return buf
        key = (name, buf.data_ptr(), buf.dtype, buf._version)
        cache = self.__dict__.setdefault("_fp32_cache", {})
        hit = cache.get(name)
        if hit is None or hit[0] != key:
            hit = (key, buf.float())
            cache[name] = hit
        return hit[1]

    def _lb_coef(self, device) -> torch.Tensor:
        cache = self.__dict__.setdefault("_lb_coef_cache", {})
        t = cache.get(device)
        if t is None:
            t = torch.tensor(self._lb_coef_values, dtype=torch.float32, device=device)
            cache[device] = t
        return t

    def _aux_stream(self, device) -> torch.cuda.Stream:
        """Side stream the auxiliary-loss kernel runs on (one per module and
        device), so that it overlaps the routing and the expert GEMMs."""
        cache = self.__dict__.setdefault("_aux_stream_cache", {})
        s = cache.get(device)
        if s is None:
            s = torch.cuda.Stream(device=device)
            cache[device] = s
        return s

    def _route_weights(self, x_flat, overlap: bool = False):
        """(logits, probs, top-k weights, selected int32, lse, (losses, f_i, z)),
        the auxiliary losses from the router head's own selection counts (f_i in
        x's dtype).  overlap: the loss kernel runs on the side stream; the caller
        must join it (`_join_aux`) before using the loss values."""
        router_logits = self.router(x_flat)
        router_probs, top_k_weights, selected, lse, losses, f_i, z = _RouterHead.apply(
            router_logits, self.num_active_experts, self.norm_topk_prob, x_flat.dtype,
            self._fp32("expert_widths_normalized"), self._lb_coef(x_flat.device),
            self._aux_stream(x_flat.device) if overlap else None)
        return router_logits, router_probs, top_k_weights, selected, lse, (losses, f_i, z)

    def _join_aux(self, device) -> None:
        torch.cuda.current_stream(device).wait_stream(self._aux_stream(device))

    def _aux_losses(self, router_logits, lse, head_losses, router_probs):
        losses, f_i, z = head_losses
        z, lb, cl, f_i = _AuxLosses.apply(router_logits, router_probs, lse, losses, f_i, z,
                                          self._lb_coef(router_logits.device),
                                          self._fp32("expert_widths_normalized"))
        aux = {"router_z_loss": z, "load_balance_loss": lb, "compute_loss": cl}
        return aux, f_i

    # ------------------------------------------------------------------ forward
    @torch.compiler.disable
    def forward(self, x: torch.Tensor):
        """x: [batch, seq, n_embd] -> (output, aux_loss dict, f_i)."""
        batch_size, seq_len, n_embd = x.shape
        x_flat = x.reshape(batch_size * seq_len, n_embd)
        router_logits, router_probs, top_k_weights, selected, lse, head_losses = (
            self._route_weights(x_flat, overlap=True))
        out_flat, tokens_per_expert = _MoEMLPFunction.apply(
            x_flat.to(self.w1.dtype), self.w1, self.w2, top_k_weights.reshape(-1),
            selected.reshape(-1), self._plan(),
        )
        output = out_flat.reshape(batch_size, seq_len, -1)
        self._join_aux(x.device)
        aux, f_i = self._aux_losses(router_logits, lse, head_losses, router_probs)
        return output, aux, f_i

    def _offsets(self, padded_bins, device):
        expert_token_offsets = torch.cat(
            [torch.zeros(1, device=device, dtype=torch.int32), padded_bins])
        padded_tokens_per_expert = torch.cat([padded_bins[:1], padded_bins[1:] - padded_bins[:-1]])
        return expert_token_offsets, padded_tokens_per_expert

    def forward_with_intermediates(self, x: torch.Tensor) -> dict[str, Any]:
        """Forward returning every intermediate in the reference layout (moe.py:305-409)."""
        batch_size, seq_len, n_embd = x.shape
        x_flat = x.reshape(batch_size * seq_len, n_embd)
        router_logits, router_probs, top_k_weights, selected_experts, _, _ = self._route_weights(
            x_flat)
        selected_experts = selected_experts.long()  # torch.topk's index dtype
        top_k_weights_flat = top_k_weights.reshape(-1)
        selected_experts_flat = selected_experts.reshape(-1)
        bin_ids, indices, tokens_per_expert, bins, padded_bins = fused_route(
            selected_experts_flat, self.num_experts, block_size=self.block_size, rounding="up")
        expert_token_offsets, padded_tokens_per_expert = self._offsets(padded_bins, x.device)
        x_gathered = padded_gather(x_flat, indices, bin_ids, bins, padded_bins,
                                   self.num_active_experts)
        x_up = grouped_gemm_up(x_gathered.to(self.w1.dtype), self.w1, expert_token_offsets,
                               self.expert_weight_offsets_t, self.expert_widths_t,
                               padded_tokens_per_expert, self.max_expert_width,
                               activation="relu_squared")
        x_down = grouped_gemm_down(x_up, self.w2, expert_token_offsets,
                                   self.expert_weight_offsets_t, self.expert_widths_t,
                                   padded_tokens_per_expert, self.config.n_embd)
        output_flat = padded_scatter(x_down, indices, bin_ids, top_k_weights_flat, bins,
                                     padded_bins, self.num_active_experts)
        output = output_flat.reshape(batch_size, seq_len, -1)
        return {
            "output": output,
            "x_flat": x_flat,
            "router_logits": router_logits,
            "router_probs": router_probs,
            "top_k_weights": top_k_weights,
            "top_k_weights_flat": top_k_weights_flat,
            "selected_experts": selected_experts,
            "selected_experts_flat": selected_experts_flat,
            "bin_ids": bin_ids,
            "indices": indices,
            "tokens_per_expert": tokens_per_expert,
            "bins": bins,
            "padded_bins": padded_bins,
            "x_gathered": x_gathered,
            "x_after_up": x_up,
            "x_after_down": x_down,
            "x_scattered": output_flat,
        }

    def forward_profiled(self, x: torch.Tensor, profiler):
        """Forward with per-step timing through `profiler.step(name)` context
        managers, with the reference's step names (moe.py:411-518)."""
        batch_size, seq_len, n_embd = x.shape
        with profiler.step("flatten"):
            x_flat = x.reshape(batch_size * seq_len, n_embd)
        with profiler.step("routing"):
            router_logits, router_probs, top_k_weights, selected_experts, lse, head_losses = (
                self._route_weights(x_flat))
            top_k_weights_flat = top_k_weights.reshape(-1)
            selected_experts_flat = selected_experts.reshape(-1)
        with profiler.step("fused_route"):
            bin_ids, indices, tokens_per_expert, bins, padded_bins = fused_route(
                selected_experts_flat, self.num_experts, block_size=self.block_size,
                rounding="up")
            expert_token_offsets, padded_tokens_per_expert = self._offsets(padded_bins, x.device)
        with profiler.step("gather"):
            x_gathered = padded_gather(x_flat, indices, bin_ids, bins, padded_bins,
                                       self.num_active_experts)
        with profiler.step("gemm_up"):
            x_up = grouped_gemm_up(x_gathered.to(self.w1.dtype), self.w1, expert_token_offsets,
                                   self.expert_weight_offsets_t, self.expert_widths_t,
                                   padded_tokens_per_expert, self.max_expert_width,
                                   activation="relu_squared")
        with profiler.step("gemm_down"):
            x_down = grouped_gemm_down(x_up, self.w2, expert_token_offsets,
                                       self.expert_weight_offsets_t, self.expert_widths_t,
                                       padded_tokens_per_expert, self.config.n_embd)
        with profiler.step("scatter"):
            output_flat = padded_scatter(x_down, indices, bin_ids, top_k_weights_flat, bins,
                                         padded_bins, self.num_active_experts)
        with profiler.step("reshape"):
            output = output_flat.reshape(batch_size, seq_len, -1)
        with profiler.step("aux_loss"):
            aux, f_i = self._aux_losses(router_logits, lse, head_losses, router_probs)
        return output, aux, f_i
