"""Host-side logic of expert parallelism, on CPU: expert placement, the
exchange plan of the C ABI (moe_ep_plan) checked by simulating where every
rank's rows land, and (gloo backend, world size 2) the sharded <-> unsharded
state_dict round trip."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def test_shard_experts_balances_each_width_group():
    from moe_b200.ep import shard_experts

    sizes = [(32, 2048), (64, 1024), (32, 512)]
    for world in (1, 2, 4, 8):
        owners = shard_experts(sizes, world)
        assert sorted(e for o in owners for e in o) == list(range(128))
        for lo, hi in ((0, 32), (32, 96), (96, 128)):
            per = [sum(lo <= e < hi for e in o) for o in owners]
            assert max(per) - min(per) <= 1
    owners = shard_experts([(4, 512), (8, 256), (4, 128)], 8)
    assert all(len(o) == 2 for o in owners)


def test_shard_experts_by_load():
    """Load-balanced placement: every expert once, every rank at least one,
    deterministic, and the busiest rank within the longest-processing-time bound
    (average + the largest single expert's work)."""
    from moe_b200.ep import shard_experts

    sizes = [(32, 2048), (64, 1024), (32, 512)]
    widths = [w for c, w in sizes for _ in range(c)]
    g = torch.Generator().manual_seed(3)
    loads = (torch.rand(128, generator=g) ** 4 * 1000).round()  # skewed, with ties at 0
    for world in (1, 2, 4, 8):
        owners = shard_experts(sizes, world, loads)
        assert owners == shard_experts(sizes, world, loads.tolist())
        assert sorted(e for o in owners for e in o) == list(range(128))
        assert all(len(o) > 0 for o in owners) and all(o == sorted(o) for o in owners)
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


def _plan(world, rank, C, E, block, owner, counts):
    import numpy as np

    from moe_b200._lib import lib

    el = int((owner == rank).sum())
    src_off = np.zeros((C, E), np.int64)
    tok_off = np.zeros(el + 1, np.int32)
    chunk_off = np.zeros((C, el + 1), np.int32)
    chunk_rows = np.zeros((C, el), np.int32)
    recv_off = np.zeros((world, C, el), np.int64)
    rc = lib.moe_ep_plan(world, rank, C, E, block, owner.ctypes.data, counts.ctypes.data,
                         src_off.ctypes.data, tok_off.ctypes.data, chunk_off.ctypes.data,
                         chunk_rows.ctypes.data, recv_off.ctypes.data)
    assert rc == 0
    return src_off, tok_off, chunk_off, chunk_rows, recv_off


@pytest.mark.parametrize("world,C,E,block", [(1, 1, 4, 16), (2, 3, 6, 16), (4, 2, 16, 16),
                                             (8, 4, 128, 16), (3, 2, 5, 64)])
def test_exchange_plan_places_every_row(world, C, E, block):
    """moe_ep_plan on every rank, then the destination the dispatch kernel
    computes for each source row (its expert-sorted row i of chunk c, expert e:
    row i - src_off[c][e] + owner's recv_off[source][c][e]), simulated on the
    host: every (source, chunk, expert) row lands in its owner's layout inside
    its expert's region and its chunk's block, in source order, with no
    overlap; blocks are padded to the block size, regions hold the chunks'
    blocks in order, and the combine reads each row back from the same place."""
    import numpy as np

    rng = np.random.default_rng(world * 100 + C * 10 + E)
    owner = rng.integers(0, world, E).astype(np.int32)
    owner[:world] = np.arange(world)  # every rank owns an expert
    counts = rng.integers(0, 40, (world, C, E)).astype(np.int32)
    counts[rng.random((world, C, E)) < 0.2] = 0  # empty blocks
    plans = [_plan(world, r, C, E, block, owner, counts) for r in range(world)]
    local = [[e for e in range(E) if owner[e] == d] for d in range(world)]
    layouts = [np.full(int(plans[d][1][-1]), -1, np.int64) for d in range(world)]
    for s in range(world):
        src_off = plans[s][0]
        for c in range(C):
            assert src_off[c, 0] == 0
            assert np.array_equal(np.diff(src_off[c]), counts[s, c, :-1])
            for e in range(E):
                d = owner[e]
                li = local[d].index(e)
                n = int(counts[s, c, e])
                dest = plans[d][4][s, c, li] + np.arange(n)  # = i + delta[e]
                _, tok_off, chunk_off, chunk_rows, _ = plans[d]
                if n:
                    assert chunk_off[c, li] <= dest[0] and dest[-1] < chunk_off[c, li] + chunk_rows[c, li]
                    assert tok_off[li] <= dest[0] and dest[-1] < tok_off[li + 1]
                assert np.all(layouts[d][dest] == -1)
                layouts[d][dest] = (s * C + c) * 10**6 + src_off[c, e] + np.arange(n)
    for d in range(world):
        _, tok_off, chunk_off, chunk_rows, _ = plans[d]
        assert tok_off[0] == 0 and np.all(np.diff(tok_off) % block == 0)
        for li, e in enumerate(local[d]):
            pos = tok_off[li]
            for c in range(C):
                assert chunk_off[c, -1] == tok_off[-1]
                tot = int(counts[:, c, e].sum())
                assert chunk_off[c, li] == pos
                assert chunk_rows[c, li] == (tot + block - 1) // block * block
                blk = layouts[d][pos : pos + chunk_rows[c, li]]
                assert np.all(blk[:tot] >= 0) and np.all(blk[tot:] == -1)
                # sources in rank order inside the block
                assert np.all(np.diff(blk[:tot] // 10**6) >= 0)
                pos += chunk_rows[c, li]
            assert pos == tok_off[li + 1]


def test_exchange_plan_rejects_bad_arguments():
    import numpy as np

    from moe_b200._lib import lib

    owner = np.array([0, 2], np.int32)  # rank 2 of a world of 2
    counts = np.zeros((2, 1, 2), np.int32)
    z = np.zeros(8, np.int64)
    t = np.zeros(8, np.int32)
    rc = lib.moe_ep_plan(2, 0, 1, 2, 16, owner.ctypes.data, counts.ctypes.data, z.ctypes.data,
                         t.ctypes.data, t.ctypes.data, t.ctypes.data, z.ctypes.data)
    assert rc == -1


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
        from moe_b200.ep import ExpertParallelMoEMLP

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
