"""Device timeline of one expert-parallel training step of bench.py's c5
layer, printed by rank 0: every kernel of this package (GEMMs, the exchange's
dispatch / combine) with its start, end and duration in ms from the step's
start, measured with CUDA events on the stream it ran on.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \
        --master-addr 127.0.0.1 --master-port 29533 \
        triton-variable-moe_b200/ep_timeline.py        (CHUNKS=4 by default)
"""
import os, sys, copy
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))
import torch, torch.distributed as dist
import bench
from moe_b200.kernels import _ops
ws, rank, local = bench.dist_env()
torch.cuda.set_device(local); dev = torch.device("cuda", local)
torch.cuda.set_stream(torch.cuda.Stream(device=dev))
dist.init_process_group("nccl", device_id=dev)
cfg = dict(bench.CONFIGS["c5"])
full = bench.build_layer(cfg, dev)
x_h, g_h = bench.make_tokens(cfg, rank)
x = x_h.to(dev)
from moe_b200 import TritonMoEConfig
from moe_b200.ep import ExpertParallelMoEMLP, measure_expert_loads
mcfg = TritonMoEConfig(n_embd=cfg["n_embd"], expert_sizes=cfg["expert_sizes"], num_active_experts=cfg["top_k"], block_size=64)
loads = measure_expert_loads(full.router, x, cfg["top_k"])
with torch.device(dev):
    layer = ExpertParallelMoEMLP(mcfg, expert_loads=loads, chunks=int(os.environ.get("CHUNKS", "4")))
layer.router = copy.deepcopy(full.router)
layer.load_full_state_dict(full.state_dict())
layer = layer.to(dev, torch.bfloat16)
del full; torch.cuda.empty_cache()
xr = x.requires_grad_(True); gout = g_h.to(dev)
def step():
    layer.zero_grad(set_to_none=True); xr.grad = None
    out, _, _ = layer(xr); out.backward(gout)
for _ in range(3): step()
torch.cuda.synchronize(); dist.barrier()
t0 = torch.cuda.Event(enable_timing=True); t0.record()
with _ops.record_kernel_events() as evs:
    step()
t1 = torch.cuda.Event(enable_timing=True); t1.record()
torch.cuda.synchronize()
if rank == 0:
    rows = sorted([(n, t0.elapsed_time(a), t0.elapsed_time(b)) for n, a, b in evs], key=lambda r: r[1])
    print("total", t0.elapsed_time(t1))
    for n, a, b in rows:
        if b - a > 0.05: print(f"{n:32s} {a:8.2f} {b:8.2f} {b-a:7.2f}")
dist.destroy_process_group()
