"""Host-side logic of expert parallelism, on CPU with the gloo backend
(world size 2): expert placement, split sizes, the count and row exchanges,
and the sharded <-> unsharded state_dict round trip."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def test_shard_experts_balances_each_width_group():
    from moe_b200.ep import rank_major_order, shard_experts

    sizes = [(32, 2048), (64, 1024), (32, 512)]
    for world in (1, 2, 4, 8):
        owners = shard_experts(sizes, world)
        assert sorted(e for o in owners for e in o) == list(range(128))
        for lo, hi in ((0, 32), (32, 96), (96, 128)):
            per = [sum(lo <= e < hi for e in o) for o in owners]
            assert max(per) - min(per) <= 1
        assert sorted(rank_major_order(owners)) == list(range(128))
    owners = shard_experts([(4, 512), (8, 256), (4, 128)], 8)
    assert all(len(o) == 2 for o in owners)


def test_shard_experts_by_load():
    """Load-balanced placement: every expert once, every rank at least one,
    deterministic, and the busiest rank within the longest-processing-time bound
    (average + the largest single expert's work)."""
    from moe_b200.ep import rank_major_order, shard_experts

    sizes = [(32, 2048), (64, 1024), (32, 512)]
    widths = [w for c, w in sizes for _ in range(c)]
    g = torch.Generator().manual_seed(3)
    loads = (torch.rand(128, generator=g) ** 4 * 1000).round()  # skewed, with ties at 0
    for world in (1, 2, 4, 8):
        owners = shard_experts(sizes, world, loads)
        assert owners == shard_experts(sizes, world, loads.tolist())
        assert sorted(e for o in owners for e in o) == list(range(128))
        assert all(len(o) > 0 for o in owners) and all(o == sorted(o) for o in owners)
        assert sorted(rank_major_order(owners)) == list(range(128))
        work = [float(loads[e]) * widths[e] for e in range(128)]
        per = [sum(work[e] for e in o) for o in owners]
        assert max(per) <= sum(work) / world + max(work) + 1e-6
        rr = shard_experts(sizes, world)
        rr_per = [sum(work[e] for e in o) for o in rr]
        assert max(per) <= max(rr_per) + 1e-6
    # one hot expert: it gets a rank of its own
    hot = [0.0] * 8
    hot[5] = 100.0
    owners = shard_experts([(8, 64)], 4, hot)
    assert [5] in owners and all(len(o) > 0 for o in owners)
    with pytest.raises(ValueError):
        shard_experts([(8, 64)], 2, [1.0] * 7)
    with pytest.raises(ValueError):
        shard_experts([(8, 64)], 2, [-1.0] + [1.0] * 7)


def test_split_sizes():
    from moe_b200.ep import split_sizes

    counts = torch.tensor([3, 0, 5, 1, 2])
    assert split_sizes(counts, [2, 3]) == [3, 8]
    assert split_sizes(counts, [1, 1, 3]) == [3, 0, 8]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from moe_b200 import TritonMoEConfig, TritonMoEMLP
        from moe_b200.ep import ExpertParallelMoEMLP, exchange_counts, exchange_rows, split_sizes

        # count exchange: rank r has counts c[r][e] for rank-major experts
        experts_per_rank = [2, 3]
        counts = torch.tensor([rank * 10 + e for e in range(5)], dtype=torch.int32)
        recv = exchange_counts(counts, experts_per_rank, rank, None)
        lo = [0, 2][rank]
        want = torch.tensor([[src * 10 + e for e in range(lo, lo + experts_per_rank[rank])]
                             for src in range(world)], dtype=torch.int32)
        assert torch.equal(recv, want), (recv, want)
        # row exchange: rows tagged with (source, position)
        send = split_sizes(counts, experts_per_rank)
        rows = torch.arange(sum(send), dtype=torch.float32)[:, None] + 1000 * rank
        got = exchange_rows(rows.repeat(1, 3), send, recv.sum(1).tolist(), None)
        parts = []
        for src in range(world):
            src_counts = torch.tensor([src * 10 + e for e in range(5)])
            s_send = split_sizes(src_counts, experts_per_rank)
            start = sum(s_send[:rank])
            parts.append(torch.arange(start, start + s_send[rank], dtype=torch.float32) + 1000 * src)
        assert torch.equal(got[:, 0], torch.cat(parts))
        # sharded module: full state_dict round trip
        torch.manual_seed(0)
        cfg = TritonMoEConfig(n_embd=32, expert_sizes=[(2, 64), (3, 32)], num_active_experts=2,
                              block_size=16)
        ref = TritonMoEMLP(cfg)
        ep = ExpertParallelMoEMLP(cfg)
        ep.load_full_state_dict(ref.state_dict())
        full = ep.full_state_dict()
        for key in ("router.weight", "w1", "w2"):
            assert torch.equal(full[key], ref.state_dict()[key]), key
        assert ep.w1.shape[1] == sum(ep.expert_widths[e] for e in ep.local_experts)
        # measured loads are summed over the ranks; a placement from them
        # round-trips the state_dict too
        from moe_b200.ep import measure_expert_loads

        x = torch.randn(64, 32, generator=torch.Generator().manual_seed(rank))
        loads = measure_expert_loads(ref.router, x, 2)
        mine = torch.bincount(ref.router(x).topk(2, dim=-1).indices.reshape(-1), minlength=5)
        assert loads.shape == (5,) and float(loads.sum()) == 2 * 64 * 2
        assert bool((loads >= mine.double()).all())
        epl = ExpertParallelMoEMLP(cfg, expert_loads=loads)
        epl.load_full_state_dict(ref.state_dict())
        full = epl.full_state_dict()
        for key in ("router.weight", "w1", "w2"):
            assert torch.equal(full[key], ref.state_dict()[key]), key
        # re-placement by other loads moves the weights with their experts
        from moe_b200.ep import shard_experts

        new_loads = [1.0, 50.0, 2.0, 40.0, 3.0]
        epl.rebalance(new_loads)
        assert epl.owners == shard_experts(cfg.expert_sizes, world, new_loads)
        assert epl.local_experts == epl.owners[rank]
        assert epl.w1.shape[1] == sum(epl.expert_widths[e] for e in epl.local_experts)
        assert int(epl.local_weight_offsets[-1]) == epl.w1.shape[1]
        full = epl.full_state_dict()
        for key in ("router.weight", "w1", "w2"):
            assert torch.equal(full[key], ref.state_dict()[key]), key
        assert sorted(epl.global_of_rank_major.tolist()) == list(range(5))
        q.put((rank, "ok"))
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


def test_ep_exchange_and_state_dict_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
