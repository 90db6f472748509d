"""Expert-parallel layer on 2 GPUs (NCCL) against the single-GPU layer on the
concatenated batch: same outputs and input gradients for each rank's tokens,
same weight gradients for each rank's experts (|a-b| <= 1e-2 * scale +
2e-2 |b|).  Skipped with fewer than two GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _close(a, b, what):
    a, b = a.float(), b.float()
    scale = b.abs().max().clamp_min(1e-30)
    bad = (a - b).abs() > 1e-2 * scale + 2e-2 * b.abs()
    assert not bad.any(), f"{what}: {int(bad.sum())} mismatches, max err {(a - b).abs().max():.3e}"


def _worker(rank, world, port, sizes, q, placement="round-robin"):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from moe_b200 import TritonMoEConfig, TritonMoEMLP
        from moe_b200.ep import ExpertParallelMoEMLP

        H, k, T = 256, 2, 1024
        cfg = TritonMoEConfig(n_embd=H, expert_sizes=sizes, num_active_experts=k, block_size=64)
        torch.manual_seed(0)
        ref = TritonMoEMLP(cfg)
        with torch.no_grad():
            for p in (ref.router.weight, ref.w1, ref.w2):
                p.normal_(0, 0.02)
        loads = None
        if placement == "load":  # a skewed placement: rank 0 gets the busiest experts' rows
            loads = [float((e * 7) % 5 + 1) for e in range(ref.num_experts)]
        ep = ExpertParallelMoEMLP(cfg, expert_loads=loads)
        ep.load_full_state_dict(ref.state_dict())
        ref = ref.to(dev, torch.bfloat16)
        ep = ep.to(dev, torch.bfloat16)
        g = torch.Generator(device="cpu").manual_seed(1)
        xg = torch.randn(world, T, H, generator=g).to(dev, torch.bfloat16)
        gg = torch.randn(world, T, H, generator=g).to(dev, torch.bfloat16)
        for it in range(3):  # the second step reuses every cached plan
            if it == 2:  # then re-place the experts (weights move with them)
                ep.rebalance([float(ref.num_experts - e) for e in range(ref.num_experts)])
            ep.zero_grad(set_to_none=True)
            ref.zero_grad(set_to_none=True)
            x = xg[rank : rank + 1].clone().requires_grad_()
            out, aux, f_i = ep(x)
            out.backward(gg[rank : rank + 1])
            xr = xg.reshape(1, world * T, H).clone().requires_grad_()
            out_r, _, _ = ref(xr)
            out_r.backward(gg.reshape(1, world * T, H))
            _close(out[0], out_r[0, rank * T : (rank + 1) * T], "out")
            _close(x.grad[0], xr.grad[0, rank * T : (rank + 1) * T], "dx")
            offs = [0]
            for w in ep.expert_widths:
                offs.append(offs[-1] + w)
            w1r = torch.cat([ref.w1.grad[:, offs[e]:offs[e + 1]] for e in ep.local_experts], 1)
            w2r = torch.cat([ref.w2.grad[offs[e]:offs[e + 1]] for e in ep.local_experts], 0)
            _close(ep.w1.grad, w1r, "dw1")
            _close(ep.w2.grad, w2r, "dw2")
            assert torch.isfinite(aux["router_z_loss"].float()) and f_i.shape == (ep.num_experts,)
        torch.cuda.synchronize()
        q.put((rank, "ok"))
    except Exception as exc:
        import traceback

        q.put((rank, traceback.format_exc()[-2000:]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("placement", ["round-robin", "load"])
@pytest.mark.parametrize("sizes", [[(8, 512)], [(4, 512), (8, 256), (4, 128)]])
def test_ep_matches_single_gpu_layer(sizes, placement):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, sizes, q, placement))
             for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert results == {0: "ok", 1: "ok"}, results


@pytest.mark.parametrize("placement", ["round-robin", "load"])
def test_ep_world1_matches_single_gpu_layer(placement):
    """The expert-parallel layer on one rank (NCCL world of 1: the exchanges are
    local copies) against the single-GPU layer: runs on a one-GPU machine too."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    p = ctx.Process(target=_worker, args=(0, 1, port, [(4, 512), (8, 256), (4, 128)], q,
                                          placement))
    p.start()
    results = dict([q.get(timeout=600)])
    p.join(timeout=120)
    assert results == {0: "ok"}, results
