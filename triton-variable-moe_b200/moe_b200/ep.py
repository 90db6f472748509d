"""Expert parallelism for the MoE MLP over the GPUs of one node.

The reference is single-GPU only.  Here tokens stay data-parallel (each rank
routes its own tokens with the replicated router) and experts are sharded: an
expert's weights live on exactly one rank.  One training step is

    forward  : router head -> routing in rank-major expert order -> gather
               -> all_to_all(counts) -> all_to_all(rows) -> local routing of
               the received rows -> grouped GEMM up (relu^2) -> down ->
               un-permute -> all_to_all back -> weighted top-k combine
    backward : weighted gather of dOut -> all_to_all -> local dIntermediate
               (fused relu^2') / dW2 / dX / dW1 -> all_to_all back -> combine

All compute is the package's sm_100a kernels; the exchanges are NCCL
all-to-alls (torch.distributed, backend "nccl") over NVLink/NVSwitch.  The
row counts of the exchange are read on the host once per direction (NCCL's
all-to-all takes host split sizes), so an expert-parallel step synchronises
the host once in the forward; the single-GPU layer does not.

Expert placement (`shard_experts`): by default round-robin within each
(count, width) group of the config, continuing the rank counter across
groups, so every rank gets a near-equal share of each width class
(parameters, and FLOPs under uniform routing).  Under skewed routing the
ranks that own the popular experts receive more rows, and every all-to-all
waits for the busiest rank; given measured per-expert token counts
(`expert_loads`, e.g. the all-reduced tokens_per_expert of a calibration
step), experts are placed greedily instead: in decreasing order of work
(tokens x width), each to the rank with the least work so far.
Expert-local weights are stored concatenated in the rank's local expert
order; `full_state_dict()` / `load_full_state_dict()` convert to and from the
reference's unsharded `w1`/`w2` layout.

The router weight is replicated; its gradient (from the auxiliary losses) is
local to each rank's tokens and should be all-reduced by the caller's data
parallelism, as for any replicated parameter.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.autograd.function import once_differentiable

from .kernels import _ops
from .moe import TritonMoEConfig, TritonMoEMLP, _AuxLosses, _Plan, _RouterHead


def shard_experts(expert_sizes, world_size: int, loads=None) -> list[list[int]]:
    """Global expert ids owned by each rank, ascending within a rank.

    loads None: round-robin within size groups.  loads (per-expert token
    counts, any non-negative numbers): longest-processing-time-first greedy
    placement of the work loads[e] * width[e]; the first world_size experts
    of that order go to distinct ranks, so every rank owns at least one expert
    when there are at least as many experts as ranks.  Ties (equal work, equal
    rank totals) resolve to the lower expert id and the lower rank, so every
    rank computes the same placement."""
    owners: list[list[int]] = [[] for _ in range(world_size)]
    widths = [w for count, w in expert_sizes for _ in range(count)]
    if loads is None:
        for eid in range(len(widths)):
            owners[eid % world_size].append(eid)
        return owners
    loads = [float(v) for v in (loads.tolist() if hasattr(loads, "tolist") else loads)]
    if len(loads) != len(widths) or any(not (v >= 0) for v in loads):
        raise ValueError("expert_loads needs one non-negative value per expert")
    work = [loads[e] * widths[e] for e in range(len(widths))]
    total = [0.0] * world_size
    for e in sorted(range(len(widths)), key=lambda e: (-work[e], e)):
        # ranks still without an expert first, then the least total work
        r = min(range(world_size), key=lambda j: (len(owners[j]) > 0, total[j], j))
        owners[r].append(e)
        total[r] += work[e]
    return [sorted(o) for o in owners]


def rank_major_order(owners: list[list[int]]) -> list[int]:
    """Global expert ids in rank-major order (rank 0's experts first)."""
    return [e for ids in owners for e in ids]


def split_sizes(counts_rank_major: torch.Tensor, experts_per_rank: list[int]) -> list[int]:
    """Rows to send to each rank from the per-expert counts in rank-major order."""
    out, pos = [], 0
    for n in experts_per_rank:
        out.append(int(counts_rank_major[pos : pos + n].sum()))
        pos += n
    return out


def exchange_counts(counts_rank_major: torch.Tensor, experts_per_rank: list[int], rank: int,
                    group) -> torch.Tensor:
    """all_to_all of per-expert counts: returns [world, E_local(rank)] counts of the
    rows this rank will receive from every source rank, per local expert."""
    world = len(experts_per_rank)
    e_loc = experts_per_rank[rank]
    recv = torch.empty(world * e_loc, dtype=counts_rank_major.dtype, device=counts_rank_major.device)
    dist.all_to_all_single(recv, counts_rank_major.contiguous(), output_split_sizes=[e_loc] * world,
                           input_split_sizes=list(experts_per_rank), group=group)
    return recv.view(world, e_loc)


def exchange_rows(rows: torch.Tensor, send: list[int], recv: list[int], group) -> torch.Tensor:
    out = torch.empty(sum(recv), rows.shape[1], dtype=rows.dtype, device=rows.device)
    dist.all_to_all_single(out, rows.contiguous(), output_split_sizes=recv, input_split_sizes=send,
                           group=group)
    return out


@dataclass
class _EPPlan:
    group: object
    world: int
    rank: int
    num_experts: int
    top_k: int
    block_size: int
    hidden: int
    experts_per_rank: list[int]
    rank_major_of_global: torch.Tensor  # [E] int64: global id -> rank-major position
    global_of_rank_major: torch.Tensor  # [E] int64
    local: _Plan  # plan of the local grouped GEMMs (top_k = 1 over received rows)


class _EPMoEFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_flat, w1, w2, weights, selected, plan: _EPPlan):
        ctx.set_materialize_grads(False)  # no zero-filled grads for unused outputs
        T, H = x_flat.shape
        k, E = plan.top_k, plan.num_experts
        dev, dt = x_flat.device, x_flat.dtype
        lp = plan.local
        # 1. routing in rank-major expert order, no padding (block 1)
        sel_rm = plan.rank_major_of_global[selected.long()]
        r = _ops.route(sel_rm, E, 1, "up")
        A = T * k
        xs = torch.empty(max(A, 1), H, device=dev, dtype=dt)
        _ops.gather(x_flat, r.row_to_assignment, k, A, out=xs)
        # 2. counts, then rows, to the owning ranks (one host read of the sizes)
        recv_counts = exchange_counts(r.tokens_per_expert, plan.experts_per_rank, plan.rank,
                                      plan.group)
        sizes = torch.cat([r.tokens_per_expert, recv_counts.reshape(-1)]).cpu()
        send = split_sizes(sizes[:E], plan.experts_per_rank)
        rc = sizes[E:].view(plan.world, -1)
        recv = [int(v) for v in rc.sum(1)]
        R = sum(recv)
        xr = exchange_rows(xs[:A], send, recv, plan.group)
        # 3. local routing of the received rows (their local expert ids)
        e_loc = lp.num_experts
        local_ids = torch.arange(e_loc, device=dev, dtype=torch.int32).repeat(plan.world)
        sel_r = torch.repeat_interleave(local_ids, rc.reshape(-1).to(dev), output_size=R)
        lr = _ops.route(sel_r, e_loc, lp.block_size, "up")
        cap = max(lr.p_capacity, 1)
        p_dev = lr.expert_token_offsets[e_loc:]
        train = any(ctx.needs_input_grad[:3])
        xg = torch.empty(cap, H, device=dev, dtype=dt)
        src = xr if R > 0 else torch.zeros(1, H, device=dev, dtype=dt)
        _ops.gather(src, lr.row_to_assignment, 1, lr.p_capacity, out=xg, rows_device=p_dev)
        h = torch.empty(cap, lp.max_width, device=dev, dtype=dt)
        pre = torch.empty_like(h) if train else None
        # up (relu^2) and down in one launch, as in the single-GPU layer
        y = torch.empty(cap, H, device=dev, dtype=dt)
        _ops.gemm_up_down(xg, w1, w2, lr.expert_token_offsets, lp.w_off, None, e_loc, h, pre, y,
                          tile_n_width=lp.tile_n_width, tile_n_hidden=lp.tile_n_hidden)
        y_recv = _ops.combine(y, lr.assignment_to_row, R, 1, weights=None)
        # 4. results back to the source ranks, weighted combine of the k copies
        ys = exchange_rows(y_recv, recv, send, plan.group)
        out = _ops.combine(ys, r.assignment_to_row, T, k, weights=weights)
        if train:
            ctx.save_for_backward(xg, h, pre, weights, w1, w2, r.row_to_assignment,
                                  r.assignment_to_row, lr.row_to_assignment,
                                  lr.assignment_to_row, lr.expert_token_offsets)
            ctx.plan, ctx.send, ctx.recv, ctx.T, ctx.R, ctx.cap = plan, send, recv, T, R, lr.p_capacity
        tpe_global = r.tokens_per_expert[plan.rank_major_of_global]
        ctx.mark_non_differentiable(tpe_global)
        return out, tpe_global

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out, _g_tpe):
        if grad_out is None:
            return None, None, None, None, None, None
        (xg, h, pre, weights, w1, w2, r2a, a2r, lr2a, la2r, ltok) = ctx.saved_tensors
        plan = ctx.plan
        lp = plan.local
        k, e_loc = plan.top_k, lp.num_experts
        T, R, cap = ctx.T, ctx.R, ctx.cap
        A = T * k
        dev, dt = xg.device, xg.dtype
        H = xg.shape[1]
        grad_out = grad_out.to(dt)
        gys = torch.empty(max(A, 1), H, device=dev, dtype=dt)
        _ops.gather(grad_out, r2a, k, A, out=gys, weights=weights)
        gyr = exchange_rows(gys[:A], ctx.send, ctx.recv, plan.group)
        rows = max(cap, 1)
        p_dev = ltok[e_loc:]
        gy = torch.empty(rows, H, device=dev, dtype=dt)
        src = gyr if R > 0 else torch.zeros(1, H, device=dev, dtype=dt)
        _ops.gather(src, lr2a, 1, cap, out=gy, rows_device=p_dev)
        dact = torch.empty(rows, lp.max_width, device=dev, dtype=dt)
        gw2 = torch.empty_like(w2)
        _ops.gemm_down_backward(gy, h, w2, ltok, lp.w_off, None, e_loc, dact, gw2, pre_act=pre,
                                tile_n_width=lp.tile_n_width, tile_n_hidden=lp.tile_n_hidden)
        gw1 = torch.empty_like(w1)
        gxg = torch.empty(rows, H, device=dev, dtype=dt) if ctx.needs_input_grad[0] else None
        _ops.gemm_up_backward(dact, xg, w1, ltok, lp.w_off, None, e_loc, gxg, gw1,
                              tile_n_width=lp.tile_n_width, tile_n_hidden=lp.tile_n_hidden)
        gx = None
        if gxg is not None:
            gx_recv = _ops.combine(gxg, la2r, R, 1, weights=None)
            gxs = exchange_rows(gx_recv, ctx.recv, ctx.send, plan.group)
            gx = _ops.combine(gxs, a2r, T, k, weights=None)
        return gx, gw1, gw2, None, None, None


@torch.no_grad()
def measure_expert_loads(router: nn.Module, x: torch.Tensor, top_k: int, group=None) -> torch.Tensor:
    """Tokens routed to each expert by `router` over this rank's tokens x
    [..., n_embd], summed over the ranks of `group` (collective): the
    expert_loads of a load-balanced placement.  top-k of the logits is the
    top-k of the sigmoid probabilities the layer routes on."""
    logits = router(x.reshape(-1, x.shape[-1]))
    sel = logits.float().topk(top_k, dim=-1).indices.reshape(-1)
    counts = torch.bincount(sel, minlength=logits.shape[-1]).to(torch.float64)
    if dist.is_initialized():
        dist.all_reduce(counts, group=group)
    return counts.cpu()


class ExpertParallelMoEMLP(nn.Module):
    """TritonMoEMLP with its experts sharded over the ranks of `group`.

    Construct it on every rank with the same config and seed; each rank keeps
    the experts `shard_experts` gives it.  forward(x) takes this rank's tokens
    [batch, seq, n_embd] and returns (output, aux_loss, f_i) like
    TritonMoEMLP, with the auxiliary losses and f_i computed over this rank's
    tokens.  expert_loads (the same on every rank; see `measure_expert_loads`)
    switches the expert placement from round-robin to load-balanced.
    """

    def __init__(self, config: TritonMoEConfig, group=None, expert_loads=None):
        super().__init__()
        if not dist.is_initialized():
            raise RuntimeError("ExpertParallelMoEMLP needs an initialised torch.distributed group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        full = TritonMoEMLP(config)  # same init as the single-GPU layer
        self.config = config
        self.num_experts = full.num_experts
        self.num_active_experts = full.num_active_experts
        self.norm_topk_prob = full.norm_topk_prob
        self.block_size = full.block_size
        self.expert_widths = full.expert_widths
        self.router = full.router
        self.register_buffer("expert_widths_normalized", full.expert_widths_normalized.clone(),
                             persistent=False)
        self._lb_coef_values = full._lb_coef_values
        self._place(shard_experts(config.expert_sizes, self.world, expert_loads),
                    full.w1.data, full.w2.data)

    def _place(self, owners, w1_full: torch.Tensor, w2_full: torch.Tensor) -> None:
        """Adopt an expert placement: this rank's expert weights sliced from the
        unsharded w1 / w2, and the id maps and offsets the forward uses."""
        if any(len(o) == 0 for o in owners):
            raise ValueError("every rank needs at least one expert")
        self.owners = owners
        self.local_experts = owners[self.rank]
        w1, w2 = self._slice(w1_full, w2_full)
        self.w1 = nn.Parameter(w1)
        self.w2 = nn.Parameter(w2)
        dev = w1.device
        order = rank_major_order(owners)
        inv = [0] * self.num_experts
        for pos, e in enumerate(order):
            inv[e] = pos
        self.register_buffer("rank_major_of_global",
                             torch.tensor(inv, dtype=torch.long, device=dev), persistent=False)
        self.register_buffer("global_of_rank_major",
                             torch.tensor(order, dtype=torch.long, device=dev), persistent=False)
        lw = [self.expert_widths[e] for e in self.local_experts]
        loff = [0]
        for w in lw:
            loff.append(loff[-1] + w)
        self.register_buffer("local_weight_offsets",
                             torch.tensor(loff, dtype=torch.int32, device=dev), persistent=False)
        self._local_widths = lw
        self._plan_cache: _EPPlan | None = None

    def rebalance(self, expert_loads) -> None:
        """Re-place the experts by new loads (collective: every rank calls it with
        the same loads, e.g. from `measure_expert_loads`).  The weights move with
        their experts; w1 and w2 become new Parameters (rebuild the optimizer over
        them), and gradients are dropped."""
        owners = shard_experts(self.config.expert_sizes, self.world, expert_loads)
        full = self.full_state_dict()
        dtype = self.w1.dtype
        self._place(owners, full["w1"].to(dtype), full["w2"].to(dtype))

    def _lb_coef(self, device) -> torch.Tensor:
        return TritonMoEMLP._lb_coef(self, device)


    def _slice(self, w1_full: torch.Tensor, w2_full: torch.Tensor):
        offs = [0]
        for w in self.expert_widths:
            offs.append(offs[-1] + w)
        cols = [w1_full[:, offs[e] : offs[e + 1]] for e in self.local_experts]
        rows = [w2_full[offs[e] : offs[e + 1]] for e in self.local_experts]
        return torch.cat(cols, 1).contiguous(), torch.cat(rows, 0).contiguous()

    def load_full_state_dict(self, sd: dict) -> None:
        """Load the reference's unsharded state_dict (router.weight, w1, w2)."""
        with torch.no_grad():
            self.router.weight.copy_(sd["router.weight"])
            w1, w2 = self._slice(sd["w1"].to(self.w1.device), sd["w2"].to(self.w2.device))
            self.w1.copy_(w1)
            self.w2.copy_(w2)

    def full_state_dict(self) -> dict:
        """Unsharded state_dict in the reference layout (collective: all ranks call it)."""
        H = self.config.n_embd
        offs = [0]
        for w in self.expert_widths:
            offs.append(offs[-1] + w)
        TW = offs[-1]
        w1 = torch.zeros(H, TW, dtype=self.w1.dtype, device=self.w1.device)
        w2 = torch.zeros(TW, H, dtype=self.w2.dtype, device=self.w2.device)
        lo = 0
        for e in self.local_experts:
            w = self.expert_widths[e]
            w1[:, offs[e] : offs[e + 1]] = self.w1.data[:, lo : lo + w]
            w2[offs[e] : offs[e + 1]] = self.w2.data[lo : lo + w]
            lo += w
        # each column block is non-zero on exactly one rank: a sum assembles it
        dist.all_reduce(w1, group=self.group)
        dist.all_reduce(w2, group=self.group)
        return {"router.weight": self.router.weight.data.clone(), "w1": w1, "w2": w2}

    def _plan(self) -> _EPPlan:
        p = self._plan_cache
        if p is None or p.local.w_off is not self.local_weight_offsets:
            lw = self._local_widths
            tn_w = 256 if max(lw, default=0) > 128 else 128
            tn_h = 256 if self.config.n_embd % 256 == 0 else 128
            local = _Plan(len(lw), 1, self.block_size, self.config.n_embd, max(lw),
                          self.local_weight_offsets, tn_w, tn_h)
            p = _EPPlan(self.group, self.world, self.rank, self.num_experts,
                        self.num_active_experts, self.block_size, self.config.n_embd,
                        [len(o) for o in self.owners], self.rank_major_of_global,
                        self.global_of_rank_major, local)
            self._plan_cache = p
        return p

    @torch.compiler.disable
    def forward(self, x: torch.Tensor):
        B, S, H = x.shape
        x_flat = x.reshape(B * S, H)
        logits = self.router(x_flat)
        wn = self.expert_widths_normalized.float()
        # the auxiliary losses use this rank's token counts per expert, which the
        # router head counts itself from its selections
        probs, w, sel, lse, losses, f_i, z = _RouterHead.apply(
            logits, self.num_active_experts, self.norm_topk_prob, x_flat.dtype, wn,
            self._lb_coef(logits.device), None)
        out_flat, _tpe = _EPMoEFunction.apply(x_flat.to(self.w1.dtype), self.w1, self.w2,
                                              w.reshape(-1), sel.reshape(-1), self._plan())
        z, lb, cl, f_i = _AuxLosses.apply(logits, probs, lse, losses, f_i, z,
                                          self._lb_coef(logits.device), wn)
        aux = {"router_z_loss": z, "load_balance_loss": lb, "compute_loss": cl}
        return out_flat.reshape(B, S, -1), aux, f_i
