"""Expert parallelism for the MoE MLP over the GPUs of one node.

The reference is single-GPU only.  Here tokens stay data-parallel (each rank
routes its own tokens with the replicated router) and experts are sharded: an
expert's weights live on exactly one rank.  One training step is

    forward  : router head -> per token chunk: routing of the chunk's
               assignments (expert-sorted, block size 1) -> dispatch: each
               row pushed straight into its expert owner's padded
               expert-contiguous layout over NVLink (the gather, fused) ->
               grouped GEMM up (relu^2) + down on the owner -> combine: each
               token's weighted top-k sum pulled from the owners' outputs
               over NVLink (the scatter, fused)
    backward : per chunk: weighted output gradients pushed to the owners ->
               dIntermediate (fused relu^2') and dX -> dX rows pulled back and
               summed; then dW2 and dW1 over all chunks' rows

The exchange kernels are this package's own (moe_ep_dispatch /
moe_ep_combine) on an exchange stream, over owner-layout buffers every rank
maps through CUDA IPC (moe_ep_buffer_create / _open), with one-word NCCL
all-reduces as barriers that order the ranks' accesses to each other's
buffers.  Chunk c's transfers overlap the GEMMs of its neighbours: the
dispatches of all chunks are queued first, each chunk's GEMMs wait only for
its own rows, and each chunk's combine waits only for that chunk's GEMMs on
every owner.  The GEMMs then run on fewer persistent CTAs (all SMs but
`comm_sms`; by default 8 on two ranks and 16 on more, where most rows cross
NVLink): a GEMM block holds nearly all of an SM's shared memory, so the
exchange kernels need SMs of their own.  The per-(rank,
chunk, expert) row counts are all-gathered and read on the host once per
forward (the exchange plan); the backward reuses them.

Expert placement (`shard_experts`): by default round-robin within each
(count, width) group of the config, continuing the rank counter across
groups, so every rank gets a near-equal share of each width class
(parameters, and FLOPs under uniform routing).  Under skewed routing the
ranks that own the popular experts receive more rows, and every exchange
waits for the busiest rank; given measured per-expert token counts
(`expert_loads`, e.g. the all-reduced tokens_per_expert of a calibration
step), experts are placed greedily instead: in decreasing order of work
(tokens x width), each to the rank with the least work so far.
Expert-local weights are stored concatenated in the rank's local expert
order (ascending global id); `full_state_dict()` / `load_full_state_dict()`
convert to and from the reference's unsharded `w1`/`w2` layout.

The router weight is replicated; its gradient (from the auxiliary losses) is
local to each rank's tokens and should be all-reduced by the caller's data
parallelism, as for any replicated parameter.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist
import torch.nn as nn
from torch.autograd.function import once_differentiable

from ._lib import DTYPE_CODE, check, lib, tile_ctas
from .kernels import _ops
from .moe import TritonMoEConfig, TritonMoEMLP, _AuxLosses, _RouterHead


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



def _addr(a: np.ndarray) -> int:
    return a.ctypes.data


class EPComm:
    """This package's NCCL communicator over the ranks of a torch.distributed
    group (moe_ep_comm_init), for the expert-parallel count exchange and the
    barriers that order the ranks' accesses to each other's buffers.  Created
    collectively: rank 0 makes the NCCL id, the group's own collective sends
    it to the others.  Uses the current CUDA device."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        uid = (ctypes.c_char * 128)()
        if self.rank == 0:
            check(lib.moe_ep_unique_id(ctypes.addressof(uid)), "moe_ep_unique_id")
        obj = [bytes(uid)]
        src = 0 if group is None else dist.get_global_rank(group, 0)
        dist.broadcast_object_list(obj, src=src, group=group)
        uid = (ctypes.c_char * 128).from_buffer_copy(obj[0])
        handle = ctypes.c_void_p()
        check(lib.moe_ep_comm_init(ctypes.addressof(handle), ctypes.addressof(uid), self.world,
                                   self.rank), "moe_ep_comm_init")
        self.handle = handle.value
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.word = torch.zeros(1, dtype=torch.int32, device=self.device)

    def barrier(self, stream: torch.cuda.Stream) -> None:
        check(lib.moe_ep_barrier(self.handle, self.word.data_ptr(), stream.cuda_stream),
              "moe_ep_barrier")

    def close(self) -> None:
        if self.handle:
            lib.moe_ep_comm_destroy(self.handle)
            self.handle = None


class _CudaArray:
    """__cuda_array_interface__ of raw device memory (for a torch view)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


class SharedBuffer:
    """A device buffer of this rank that every rank of the group maps (CUDA IPC
    over NVLink): `peers` is the device array of the world's base pointers the
    exchange kernels take.  Collective to create."""

    def __init__(self, comm: EPComm, nbytes: int):
        self.nbytes = int(nbytes)
        ptr = ctypes.c_void_p()
        h = (ctypes.c_char * 64)()
        check(lib.moe_ep_buffer_create(self.nbytes, ctypes.addressof(ptr), ctypes.addressof(h)),
              "moe_ep_buffer_create")
        self.ptr = ptr.value
        self.device = comm.device
        handles = [None] * comm.world
        dist.all_gather_object(handles, bytes(h), group=comm.group)
        self.opened = []
        bases = []
        for r, hb in enumerate(handles):
            if r == comm.rank:
                bases.append(self.ptr)
                continue
            hh = (ctypes.c_char * 64).from_buffer_copy(hb)
            p = ctypes.c_void_p()
            check(lib.moe_ep_buffer_open(ctypes.addressof(hh), ctypes.addressof(p)),
                  "moe_ep_buffer_open")
            self.opened.append(p.value)
            bases.append(p.value)
        self.peers = torch.tensor(bases, dtype=torch.int64, device=comm.device)

    def view(self, rows: int, cols: int, dtype: torch.dtype) -> torch.Tensor:
        """This rank's buffer as a [rows, cols] tensor (no copy)."""
        es = torch.tensor([], dtype=dtype).element_size()
        if rows * cols * es > self.nbytes:
            raise ValueError("view larger than the shared buffer")
        raw = torch.as_tensor(_CudaArray(self.ptr, (rows * cols * es // 2,), "<i2"),
                              device=self.device)
        return raw.view(dtype).view(rows, cols)

    def close(self) -> None:
        for p in self.opened:
            lib.moe_ep_buffer_close(p)
        self.opened = []
        if self.ptr:
            lib.moe_ep_buffer_free(self.ptr)
            self.ptr = 0


@dataclass
class _BufferSet:
    """The owner-layout buffers one forward/backward pair uses: x rows (the
    GEMMs' input, kept for the weight gradients), output-gradient rows, and
    output rows (the backward's dX rows reuse them)."""

    rows: int
    x: SharedBuffer
    g: SharedBuffer
    y: SharedBuffer

    def close(self) -> None:
        for b in (self.x, self.g, self.y):
            b.close()


@dataclass
class _ExchangePlan:
    """Host arrays of one step's exchange (moe_ep_plan of this rank) and the
    device tables the exchange kernels and the chunk GEMMs read."""

    counts: np.ndarray  # [world, chunks, E] int32
    tok_off: np.ndarray  # [E_loc + 1] int32: the owner layout's expert regions
    rows_needed: int  # the most rows any rank's layout needs this step
    meta: torch.Tensor  # device: tok_off | chunk_off | chunk_rows (int32)
    delta: torch.Tensor  # device [chunks, E] int64: owner-layout row - expert-sorted row
    pad: torch.Tensor  # device int64: padding rows of this rank's layout


@dataclass
class _EPState:
    """Per-layer constants of the expert-parallel forward."""

    comm: EPComm
    stream: torch.cuda.Stream  # the exchange stream
    pool: list  # free _BufferSets (same sequence of takes and returns on every rank)
    num_experts: int
    top_k: int
    hidden: int
    chunks: int
    owner: np.ndarray  # [E] int32: rank owning each global expert
    owner_dev: torch.Tensor  # [E] int32, device
    local_index: np.ndarray  # [E] int: index of each expert among its owner's experts
    local_experts: list
    w_off: torch.Tensor  # [E_loc + 1] int32, device: local weight offsets
    max_width: int
    tile_n_width: int  # N tiles with the CTA cap folded in
    tile_n_hidden: int


_LOCAL_BLOCK = 16  # rows of the owners' blocks are padded to multiples of this


def _rank_plan(st: _EPState, counts: np.ndarray, rank: int):
    world, C, E = counts.shape
    el = int((st.owner == rank).sum())
    src_off = np.zeros((C, E), np.int64)
    tok_off = np.zeros(el + 1, np.int32)
    chunk_off = np.zeros((C, el + 1), np.int32)
    chunk_rows = np.zeros((C, el), np.int32)
    recv_off = np.zeros((world, C, el), np.int64)
    check(lib.moe_ep_plan(world, rank, C, E, _LOCAL_BLOCK, _addr(st.owner), _addr(counts),
                          _addr(src_off), _addr(tok_off), _addr(chunk_off), _addr(chunk_rows),
                          _addr(recv_off)), "moe_ep_plan")
    return src_off, tok_off, chunk_off, chunk_rows, recv_off


def _make_plan(st: _EPState, counts: np.ndarray, device) -> _ExchangePlan:
    """Every rank's layout from the gathered counts: this rank's own, where its
    rows land in every owner's (delta), and the largest layout of the step."""
    world, C, E = counts.shape
    me = st.comm.rank
    counts = np.ascontiguousarray(counts, dtype=np.int32)
    plans = [_rank_plan(st, counts, d) for d in range(world)]
    src_off = plans[me][0]
    delta = np.zeros((C, E), np.int64)
    for d in range(world):
        mask = st.owner == d
        delta[:, mask] = plans[d][4][me][:, st.local_index[mask]] - src_off[:, mask]
    _, tok_off, chunk_off, chunk_rows, _ = plans[me]
    totals = counts[:, :, st.local_experts].sum(0)  # [C, E_loc] rows received per block
    lo = chunk_off[:, :-1].astype(np.int64) + totals
    hi = chunk_off[:, :-1].astype(np.int64) + chunk_rows
    idx = [np.arange(a, b, dtype=np.int64) for a, b in zip(lo.ravel(), hi.ravel()) if b > a]
    pad = np.concatenate(idx) if idx else np.zeros(0, np.int64)
    meta = np.concatenate([tok_off, chunk_off.ravel(), chunk_rows.ravel()])
    return _ExchangePlan(counts, tok_off, max(int(p[1][-1]) for p in plans),
                         torch.from_numpy(meta).to(device), torch.from_numpy(delta).to(device),
                         torch.from_numpy(pad).to(device))


def _take_buffers(st: _EPState, rows: int, row_bytes: int) -> _BufferSet:
    """A free buffer set with room for `rows` owner-layout rows (collective when
    one is created: every rank makes the same decision from the same counts)."""
    for i, bs in enumerate(st.pool):
        if bs.rows >= rows:
            return st.pool.pop(i)
    if st.pool:  # too small: replace the smallest free set
        st.pool.sort(key=lambda b: b.rows)
        st.pool.pop(0).close()
    cap = max(int(rows * 1.25), 1)
    nb = cap * row_bytes
    return _BufferSet(cap, SharedBuffer(st.comm, nb), SharedBuffer(st.comm, nb),
                      SharedBuffer(st.comm, nb))


def _after(stream_a: torch.cuda.Stream, stream_b: torch.cuda.Stream) -> None:
    """stream_a waits for the work stream_b has queued so far."""
    ev = torch.cuda.Event()
    ev.record(stream_b)
    stream_a.wait_event(ev)


def _meta_views(p: _ExchangePlan, C: int, el: int):
    tok_off = p.meta[: el + 1]
    chunk_off = p.meta[el + 1 : el + 1 + C * (el + 1)].view(C, el + 1)
    chunk_rows = p.meta[el + 1 + C * (el + 1) :].view(C, el)
    return tok_off, chunk_off, chunk_rows


def _dispatch(st, src, H, r2a, k, weights, bins, rows, delta, peers, dt, cs):
    """Push one chunk's rows (exchange stream)."""
    ev = _ops._ev_begin()
    check(lib.moe_ep_dispatch(src, H, H, r2a, k, weights, bins, rows, st.owner_dev.data_ptr(),
                              delta, peers, H, DTYPE_CODE[dt], cs.cuda_stream),
          "moe_ep_dispatch")
    _ops._ev_end(ev, "ep_dispatch")
    _ops._count(1)


def _combine(st, peers, delta, bins, a2r, tokens, k, weights, H, out, dt, cs):
    """Pull one chunk's output rows and sum them per token (exchange stream)."""
    ev = _ops._ev_begin()
    check(lib.moe_ep_combine(peers, H, st.owner_dev.data_ptr(), delta, bins, a2r, tokens, k,
                             weights, H, out, H, DTYPE_CODE[dt], cs.cuda_stream),
          "moe_ep_combine")
    _ops._ev_end(ev, "ep_combine")
    _ops._count(1)


class _EPMoEFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_flat, w1, w2, weights, selected, st: _EPState):
        ctx.set_materialize_grads(False)  # no zero-filled grads for unused outputs
        T, H = x_flat.shape
        k, E = st.top_k, st.num_experts
        # one rank has nothing to overlap: one chunk
        C = max(1, min(st.chunks if st.comm.world > 1 else 1, T))
        x_flat, weights = x_flat.contiguous(), weights.contiguous()
        dev, dt = x_flat.device, x_flat.dtype
        es = x_flat.element_size()
        comp, cs = torch.cuda.current_stream(dev), st.stream
        bounds = [T * c // C for c in range(C + 1)]
        el = len(st.local_experts)
        # 1. every chunk's assignments in expert-sorted order (block size 1)
        routes = [_ops.route(selected[bounds[c] * k : bounds[c + 1] * k], E, 1, "up")
                  for c in range(C)]
        # 2. the per-(rank, chunk, expert) counts on every rank: the one host read
        mine = torch.stack([r.tokens_per_expert for r in routes]).contiguous()
        all_counts = torch.empty(st.comm.world * C * E, dtype=torch.int32, device=dev)
        check(lib.moe_ep_gather_counts(st.comm.handle, mine.data_ptr(), all_counts.data_ptr(),
                                       C * E, comp.cuda_stream), "moe_ep_gather_counts")
        p = _make_plan(st, all_counts.view(st.comm.world, C, E).cpu().numpy(), dev)
        bs = _take_buffers(st, p.rows_needed, H * es)
        rows = max(int(p.tok_off[-1]), 1)
        _tok_off, chunk_off, chunk_rows = _meta_views(p, C, el)
        xg = bs.x.view(rows, H, dt)
        y = bs.y.view(rows, H, dt)
        if p.pad.numel():
            xg.index_fill_(0, p.pad, 0)  # padding rows: nobody pushes them
        h = torch.empty(rows, st.max_width, device=dev, dtype=dt)
        train = any(ctx.needs_input_grad[:3])
        pre = torch.empty_like(h) if train else None
        out = torch.empty(T, H, device=dev, dtype=dt)
        for t in (out, x_flat, weights, *[r.bin_ids for r in routes],
                  *[r.row_to_assignment for r in routes], *[r.assignment_to_row for r in routes]):
            t.record_stream(cs)
        # 3. exchange stream: once every rank is done with this set (barrier),
        #    push each chunk's rows into the owners' layouts, then a barrier
        _after(cs, comp)
        st.comm.barrier(cs)
        landed = []
        with torch.cuda.stream(cs):
            for c in range(C):
                r, t0, t1 = routes[c], bounds[c], bounds[c + 1]
                _dispatch(st, x_flat.data_ptr() + t0 * H * es, H, r.row_to_assignment.data_ptr(),
                          k, None, r.bin_ids.data_ptr(), (t1 - t0) * k, p.delta[c].data_ptr(),
                          bs.x.peers.data_ptr(), dt, cs)
                st.comm.barrier(cs)
                landed.append(torch.cuda.Event())
                landed[-1].record(cs)
        # 4. per chunk: the GEMMs once its rows landed; then, once every owner's
        #    GEMMs of the chunk are done (barrier), its tokens' outputs are
        #    pulled from the owners while the next chunk computes
        for c in range(C):
            comp.wait_event(landed[c])
            _ops.gemm_up_down(xg, w1, w2, chunk_off[c], st.w_off, chunk_rows[c], el, h, pre, y,
                              tile_n_width=st.tile_n_width, tile_n_hidden=st.tile_n_hidden)
            _after(cs, comp)
            st.comm.barrier(cs)
            r, t0, t1 = routes[c], bounds[c], bounds[c + 1]
            with torch.cuda.stream(cs):
                _combine(st, bs.y.peers.data_ptr(), p.delta[c].data_ptr(), r.bin_ids.data_ptr(),
                         r.assignment_to_row.data_ptr(), t1 - t0, k,
                         weights.data_ptr() + t0 * k * weights.element_size(), H,
                         out.data_ptr() + t0 * H * es, dt, cs)
        _after(comp, cs)
        if train:
            ctx.save_for_backward(h, pre, weights, w1, w2,
                                  *[r.row_to_assignment for r in routes],
                                  *[r.assignment_to_row for r in routes],
                                  *[r.bin_ids for r in routes])
            ctx.st, ctx.p, ctx.bs, ctx.bounds, ctx.C = st, p, bs, bounds, C
        else:
            st.pool.append(bs)
        tpe = routes[0].tokens_per_expert.clone()
        for r in routes[1:]:
            tpe += r.tokens_per_expert
        ctx.mark_non_differentiable(tpe)
        return out, tpe

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_out, _g_tpe):
        st, p, bs, bounds, C = ctx.st, ctx.p, ctx.bs, ctx.bounds, ctx.C
        if grad_out is None:
            st.pool.append(bs)
            return None, None, None, None, None, None
        saved = ctx.saved_tensors
        h, pre, weights, w1, w2 = saved[:5]
        r2a, a2r, bins = saved[5 : 5 + C], saved[5 + C : 5 + 2 * C], saved[5 + 2 * C : 5 + 3 * C]
        k, el = st.top_k, len(st.local_experts)
        rows, H = h.shape[0], st.hidden
        dev, dt = h.device, h.dtype
        comp, cs = torch.cuda.current_stream(dev), st.stream
        tok_off, chunk_off, chunk_rows = _meta_views(p, C, el)
        xg = bs.x.view(rows, H, dt)
        gy = bs.g.view(rows, H, dt)
        gxg = bs.y.view(rows, H, dt)  # the output rows are no longer needed
        grad_out = grad_out.to(dt).contiguous()
        es = grad_out.element_size()
        if p.pad.numel():
            gy.index_fill_(0, p.pad, 0)
        need_x = ctx.needs_input_grad[0]
        gx = torch.empty(bounds[-1], H, device=dev, dtype=dt) if need_x else None
        for t in ([gx] if need_x else []) + [grad_out]:
            t.record_stream(cs)
        # 1. each chunk's weighted output gradients pushed to the owners
        _after(cs, comp)
        st.comm.barrier(cs)
        landed = []
        with torch.cuda.stream(cs):
            for c in range(C):
                t0, t1 = bounds[c], bounds[c + 1]
                _dispatch(st, grad_out.data_ptr() + t0 * H * es, H, r2a[c].data_ptr(), k,
                          weights.data_ptr() + t0 * k * weights.element_size(),
                          bins[c].data_ptr(), (t1 - t0) * k, p.delta[c].data_ptr(),
                          bs.g.peers.data_ptr(), dt, cs)
                st.comm.barrier(cs)
                landed.append(torch.cuda.Event())
                landed[-1].record(cs)
        # 2. per chunk: dIntermediate (relu^2' fused) and dX, whose rows the
        #    sources pull while the next chunk computes; then both weight
        #    gradients over all chunks' rows, overlapping the last pulls
        dact = torch.empty(rows, st.max_width, device=dev, dtype=dt)
        for c in range(C):
            comp.wait_event(landed[c])
            _ops.gemm_down_dinter(gy, w2, chunk_off[c], st.w_off, chunk_rows[c], el, dact,
                                  pre_act=pre, tile_n=st.tile_n_width)
            if need_x:
                _ops.gemm_up_dx(dact, w1, chunk_off[c], st.w_off, chunk_rows[c], el, gxg,
                                tile_n=st.tile_n_hidden)
                _after(cs, comp)
                st.comm.barrier(cs)
                t0, t1 = bounds[c], bounds[c + 1]
                with torch.cuda.stream(cs):
                    _combine(st, bs.y.peers.data_ptr(), p.delta[c].data_ptr(), bins[c].data_ptr(),
                             a2r[c].data_ptr(), t1 - t0, k, None, H,
                             gx.data_ptr() + t0 * H * es, dt, cs)
        gw1 = gw2 = None
        if ctx.needs_input_grad[2]:
            gw2 = torch.empty_like(w2)
            _ops.gemm_down_dw(h, gy, tok_off, st.w_off, el, gw2, tile_n=st.tile_n_hidden)
        if ctx.needs_input_grad[1]:
            gw1 = torch.empty_like(w1)
            _ops.gemm_up_dw(xg, dact, tok_off, st.w_off, el, gw1, tile_n=st.tile_n_width)
        _after(comp, cs)
        st.pool.append(bs)
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
    chunks: token chunks exchanged one after another (their transfers overlap
    the GEMMs of the neighbouring chunks; one chunk on one rank); comm_sms: SMs
    the GEMMs leave to the exchange kernels (ignored on one rank).  The first
    forward creates the layer's NCCL communicator and exchange buffers
    (collective); `close()` releases them.
    """

    def __init__(self, config: TritonMoEConfig, group=None, expert_loads=None, chunks: int = 4,
                 comm_sms: int | None = None):
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
        self.chunks = max(1, int(chunks))
        if comm_sms is None:
            env = os.environ.get("MOE_EP_COMM_SMS")
            # measured at 65536 tokens per GPU (c5): 8 best at 2 ranks; 16 at 4
            # and 8 ranks, where 3/4 to 7/8 of the pulled rows cross NVLink
            comm_sms = int(env) if env else (8 if self.world <= 2 else 16)
        self.comm_sms = max(0, int(comm_sms))
        self._comm: EPComm | None = None
        self._pool: list = []  # free owner-layout buffer sets (see _take_buffers)
        self._place(shard_experts(config.expert_sizes, self.world, expert_loads),
                    full.w1.data, full.w2.data)

    def _place(self, owners, w1_full: torch.Tensor, w2_full: torch.Tensor) -> None:
        """Adopt an expert placement: this rank's expert weights sliced from the
        unsharded w1 / w2, and the offsets the forward uses."""
        if any(len(o) == 0 for o in owners):
            raise ValueError("every rank needs at least one expert")
        self.owners = owners
        self.local_experts = owners[self.rank]
        w1, w2 = self._slice(w1_full, w2_full)
        self.w1 = nn.Parameter(w1)
        self.w2 = nn.Parameter(w2)
        lw = [self.expert_widths[e] for e in self.local_experts]
        loff = [0]
        for w in lw:
            loff.append(loff[-1] + w)
        self.register_buffer("local_weight_offsets",
                             torch.tensor(loff, dtype=torch.int32, device=w1.device),
                             persistent=False)
        self._local_widths = lw
        owner = np.zeros(self.num_experts, np.int32)
        for r, ids in enumerate(owners):
            owner[ids] = r
        self._owner = owner
        self._state_cache: _EPState | None = None


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

    def close(self) -> None:
        """Release the layer's shared exchange buffers and its NCCL communicator
        (collective: every rank calls it; the layer can run again afterwards)."""
        if self._comm is not None:
            torch.cuda.synchronize(self._comm.device)
        while self._pool:
            self._pool.pop().close()
        if self._comm is not None:
            self._comm.close()
            self._comm = None
        self._state_cache = None


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


    def _state(self, device) -> _EPState:
        p = self._state_cache
        if p is None or p.w_off is not self.local_weight_offsets:
            if self._comm is None:
                with torch.cuda.device(device):
                    self._comm = EPComm(self.group)
            lw = self._local_widths
            tn_w = 256 if max(lw, default=0) > 128 else 128
            tn_h = 256 if self.config.n_embd % 256 == 0 else 128
            n_sm = torch.cuda.get_device_properties(device).multi_processor_count
            cap = max(n_sm - self.comm_sms, 1) if self.world > 1 and self.comm_sms > 0 else 0
            local_index = np.zeros(self.num_experts, np.int64)
            for ids in self.owners:
                for i, e in enumerate(ids):
                    local_index[e] = i
            p = _EPState(self._comm, torch.cuda.Stream(device=device), self._pool,
                         self.num_experts, self.num_active_experts, self.config.n_embd,
                         self.chunks, self._owner, torch.from_numpy(self._owner).to(device),
                         local_index, list(self.local_experts), self.local_weight_offsets,
                         max(lw), tn_w | tile_ctas(cap), tn_h | tile_ctas(cap))
            self._state_cache = p
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
                                              w.reshape(-1), sel.reshape(-1),
                                              self._state(x.device))
        z, lb, cl, f_i = _AuxLosses.apply(logits, probs, lse, losses, f_i, z,
                                          self._lb_coef(logits.device), wn)
        aux = {"router_z_loss": z, "load_balance_loss": lb, "compute_loss": cl}
        return out_flat.reshape(B, S, -1), aux, f_i
