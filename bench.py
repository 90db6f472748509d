"""Benchmark: MoE layer forward + backward tokens/s on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config c3]

A step is one training pass of the MoE layer over one synthetic batch:
`out, aux, f_i = layer(x); out.backward(g)` (router, routing, gather, grouped
GEMM up with relu^2, grouped GEMM down, weighted combine, and the full
backward).  The default workload (c3) is the 768-hidden variable-expert layer: n_embd=768, experts 4x512 + 8x256 + 4x128,
top-2, batch 8 x seq 1024 = 8192 tokens, bf16, x ~ N(0,1), weights N(0,0.02),
router from a random-init linear.

Execution: the layer never synchronises the host, so the step is captured once
in a CUDA graph and replayed (the eager time is reported beside it).

Timing: W untimed warm-up steps, then exactly K steps, each bracketed by CUDA
events on the launch stream, with a 256 MiB write between steps to flush the
126 MB L2; barrier + synchronize on both sides; the per-rank time is the sum
of the K step times and the job time is the max over ranks.  `value` =
tokens processed by all ranks / job time.  At N > 1 the layer is expert
parallel: every rank keeps the workload's token batch (weak scaling) and the
experts are sharded over the ranks, with NCCL all-to-all dispatch and combine;
that step runs eagerly because the exchange sizes are read on the host.

Extra keys: `roofline` (the grouped-GEMM engine: algorithmic FLOPs
12*H*sum_e n_e*w_e per step / summed device time of its launches per step (forward:
up+down in one launch; backward: dIntermediate+dX, then dW2+dW1),
against the measured bf16 peak), `cpu_baseline` (the numpy CPU oracle on the
host cores), `e2e` (pinned host input -> device, fwd+bwd, output -> host,
per step), `gpu_launches`, `clocks`.

`--impl reference` times the reference algorithm's CPU restatement (the
oracle; the reference itself is Triton/Python and cannot run on the host
outside the Triton interpreter) on the host cores for the same config and
metric.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "triton-variable-moe_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "MoE layer fwd+bwd tokens/s"

CONFIGS = {
    "c2u": dict(n_embd=256, expert_sizes=[(8, 512)], top_k=2, batch=8, seq=512, zipf=False),
    "c2v": dict(n_embd=256, expert_sizes=[(4, 512), (4, 256)], top_k=2, batch=8, seq=512, zipf=False),
    "c3": dict(n_embd=768, expert_sizes=[(4, 512), (8, 256), (4, 128)], top_k=2, batch=8, seq=1024,
               zipf=False),
    "c4": dict(n_embd=2048, expert_sizes=[(64, 1024)], top_k=8, batch=1, seq=16384, zipf=True),
    # the expert-parallel config: at N > 1 its experts are sharded over the GPUs;
    # the others run as independent replicas at N > 1 (their experts fit one GPU)
    "c5": dict(n_embd=4096, expert_sizes=[(32, 2048), (64, 1024), (32, 512)], top_k=8, batch=1,
               seq=65536, zipf=True, ep=True),
}


def workload_name(name: str, cfg: dict) -> str:
    sizes = "+".join(f"{c}x{w}" for c, w in cfg["expert_sizes"])
    return (f"{name}: MoE layer n_embd={cfg['n_embd']} experts {sizes} top-{cfg['top_k']} "
            f"tokens={cfg['batch'] * cfg['seq']}" + (" zipf(1.1) router bias" if cfg["zipf"] else ""))


def widths_of(cfg):
    return [w for c, w in cfg["expert_sizes"] for _ in range(c)]


def gemm_flops(tokens_per_expert, cfg) -> float:
    """12 * H * sum_e n_e * w_e: the six GEMMs of fwd+bwd, unpadded counts."""
    H = cfg["n_embd"]
    return float(sum(12 * H * int(n) * w for n, w in zip(tokens_per_expert, widths_of(cfg))))


def permute_bytes(cfg) -> float:
    """Unique bytes moved by gather + scatter forward and their backward mirrors."""
    T = cfg["batch"] * cfg["seq"]
    A = T * cfg["top_k"]
    H = cfg["n_embd"]
    return float(4 * (T + A) * H * 2 + 2 * A * 2)


def zipf_bias(E, seed, s=1.1):
    import torch

    g = torch.Generator().manual_seed(seed)
    ranks = torch.randperm(E, generator=g).float() + 1.0
    logp = -s * torch.log(ranks)
    logp = logp - torch.logsumexp(logp, 0)
    return logp - logp.mean()


def build_layer(cfg, device, seed=0):
    import torch

    from moe_b200 import TritonMoEConfig, TritonMoEMLP

    torch.manual_seed(seed)
    layer = TritonMoEMLP(TritonMoEConfig(n_embd=cfg["n_embd"], expert_sizes=cfg["expert_sizes"],
                                         num_active_experts=cfg["top_k"], block_size=64))
    with torch.no_grad():
        layer.router.weight.normal_(0, 0.02)
        layer.w1.normal_(0, 0.02)
        layer.w2.normal_(0, 0.02)
    if cfg["zipf"]:
        r = torch.nn.Linear(cfg["n_embd"], layer.num_experts, bias=True)
        with torch.no_grad():
            r.weight.copy_(layer.router.weight)
            r.bias.copy_(zipf_bias(layer.num_experts, seed + 1))
        layer.router = r
    return layer.to(device=device, dtype=torch.bfloat16)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, power, reasons = [], None, [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            p = [v.strip() for v in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax = float(p[2])
                power.append(float(p[3]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        loaded = [s for s, pw in zip(sm, power) if pw > 200.0] or sm
        return {
            "sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": smax,
            "reasons": sorted(reasons),
            "samples": len(sm),
            "power_w_max": max(power) if power else None,
        }


# ------------------------------------------------------------------ helpers
def gpu_selector(dev) -> str:
    """nvidia-smi -i selector (PCI bus id) of a torch device, robust to
    CUDA_VISIBLE_DEVICES renumbering."""
    import torch

    p = torch.cuda.get_device_properties(dev)
    try:
        return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except AttributeError:
        return str(dev.index)

def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def ncu_traffic(workload: str):
    """DRAM bytes per step of the grouped-GEMM launches from the committed ncu
    summary (profiles/grouped_gemm_<workload>.md, line `dram_bytes_per_step: N`)."""
    p = ROOT / "profiles" / f"grouped_gemm_{workload}.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_step:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except (ValueError, IndexError):
                return None
    return None


def cpu_oracle_step(cfg, x_np, w1, w2, sel, wts, g_np):
    from oracle import moe_oracle as orc

    orc.moe_mlp(x_np, w1, w2, sel, wts, widths_of(cfg), cfg["top_k"], 64, grad_out=g_np, dtype="bf16")


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_sample(cfg, tokens: int, seed=0):
    """Inputs for the CPU oracle on a `tokens`-token slice of the workload."""
    import numpy as np
    import torch

    layer = build_layer(cfg, "cpu", seed).float()
    g = torch.Generator().manual_seed(seed + 7)
    x = torch.randn(tokens, cfg["n_embd"], generator=g)
    with torch.no_grad():
        logits = layer.router(x.bfloat16().float())
        probs = torch.sigmoid(logits)
        w, sel = torch.topk(probs, cfg["top_k"], dim=-1)
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    gout = torch.randn(tokens, cfg["n_embd"], generator=g)
    return (x.numpy(), layer.w1.detach().numpy(), layer.w2.detach().numpy(),
            sel.reshape(-1).numpy().astype(np.int64), w.reshape(-1).numpy(), gout.numpy())


def time_cpu_oracle(cfg, budget_s=15.0, tokens=None):
    T = cfg["batch"] * cfg["seq"]
    tokens = tokens or min(T, 4096)
    args = cpu_sample(cfg, tokens)
    t0 = time.perf_counter()
    cpu_oracle_step(cfg, *args)  # warm-up (first-call allocation)
    first = time.perf_counter() - t0
    reps = max(1, min(20, int(budget_s / max(first, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(reps):
        cpu_oracle_step(cfg, *args)
    dt = (time.perf_counter() - t0) / reps
    return tokens / dt, tokens, reps


def build_ep_layer(cfg, device, seed=0, calib_x=None):
    """The same layer (same seed, same full weights) with its experts sharded over
    the ranks of the default process group.  With calib_x (this rank's tokens),
    the experts are placed by the load the router gives them over all ranks'
    tokens (ExpertParallelMoEMLP expert_loads); else round-robin."""
    import torch

    from moe_b200 import TritonMoEConfig
    from moe_b200.ep import ExpertParallelMoEMLP, measure_expert_loads

    torch.manual_seed(seed)
    mcfg = TritonMoEConfig(n_embd=cfg["n_embd"], expert_sizes=cfg["expert_sizes"],
                           num_active_experts=cfg["top_k"], block_size=64)
    full = build_layer(cfg, "cpu", seed)
    loads = None
    if calib_x is not None:
        import copy

        router = copy.deepcopy(full.router).to(device=device, dtype=calib_x.dtype)
        loads = measure_expert_loads(router, calib_x, cfg["top_k"])
        del router
    layer = ExpertParallelMoEMLP(mcfg, expert_loads=loads)
    if cfg["zipf"]:
        layer.router = full.router
    layer.load_full_state_dict({k: v.float() for k, v in full.state_dict().items()})
    return layer.to(device=device, dtype=torch.bfloat16)


def capture_step(layer, x, gout, kernel_events=False):
    """Capture one fwd+bwd of the layer in a CUDA graph (the layer never
    synchronises the host, so the whole step is capturable).  Returns the graph,
    its static output, how many of our kernels one replay launches and (with
    kernel_events) the (name, start, end) event pairs recorded around each of
    our launches inside the graph."""
    import torch

    from moe_b200.kernels import _ops

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            layer.zero_grad(set_to_none=True)
            x.grad = None
            out, _, _ = layer(x)
            out.backward(gout)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    layer.zero_grad(set_to_none=True)
    x.grad = None
    graph = torch.cuda.CUDAGraph()
    l0 = _ops.launch_count
    evs: list = []
    with torch.cuda.graph(graph):
        if kernel_events:
            with _ops.record_kernel_events(external=True) as evs:
                out, _, _ = layer(x)
                out.backward(gout)
        else:
            out, _, _ = layer(x)
            out.backward(gout)
    return graph, out, _ops.launch_count - l0, evs


# ------------------------------------------------------------------ arms
def run_reference(args, cfg, name):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    T = cfg["batch"] * cfg["seq"]
    tokens = min(T, 2048)
    xs = cpu_sample(cfg, tokens)
    for _ in range(args.warmup):
        cpu_oracle_step(cfg, *xs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_oracle_step(cfg, *xs)
    dt = time.perf_counter() - t0
    value = tokens * args.steps / dt
    cores = cpu_threads()
    sample = (f"{tokens} of the workload's {T} tokens per step (bf16-rounded fp32 numpy "
              f"restatement of the reference algorithm, fwd+bwd)")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": workload_name(name, cfg), "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_b200(args, cfg, name):
    import torch
    import torch.distributed as dist

    from moe_b200.kernels import _ops

    ws, rank, local = dist_env()
    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "error": "no CUDA device"}))
        return 1
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
        dist.init_process_group("nccl", device_id=dev)

    T = cfg["batch"] * cfg["seq"]
    H = cfg["n_embd"]
    ep = ws > 1 and cfg.get("ep", False)  # expert parallel; else one replica per GPU
    g = torch.Generator(device="cpu").manual_seed(1234 + rank)
    x_host = torch.randn(cfg["batch"], cfg["seq"], H, generator=g).to(torch.bfloat16).pin_memory()
    g_host = torch.randn(cfg["batch"], cfg["seq"], H, generator=g).to(torch.bfloat16).pin_memory()
    if ep:
        calib = x_host.to(dev) if args.placement == "load" else None
        layer = build_ep_layer(cfg, dev, seed=0, calib_x=calib)
        del calib
    else:
        layer = build_layer(cfg, dev, seed=0)
    x = x_host.to(dev).requires_grad_(True)
    gout = g_host.to(dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def step(xi, gi):
        layer.zero_grad(set_to_none=True)
        xi.grad = None
        out, aux, f_i = layer(xi)
        out.backward(gi)
        return out

    for _ in range(max(args.warmup, 3)):
        step(x, gout)
    torch.cuda.synchronize()
    if args.profile_step:
        # one eager step for an external profiler (ncu), nothing timed
        step(x, gout)
        torch.cuda.synchronize()
        return 0

    if not ep:
        graph, out_static, per_step_launches, _ = capture_step(layer, x, gout)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        run_step = graph.replay
    else:
        # expert parallel: the exchange sizes are read on the host once per step,
        # so the step runs eagerly (not captured)
        l0 = _ops.launch_count
        step(x, gout)
        torch.cuda.synchronize()
        per_step_launches = _ops.launch_count - l0
        run_step = lambda: step(x, gout)  # noqa: E731

    # clock samples: a ~1.5 s soak of the same step right before the timed loop
    sampler = ClockSampler(gpu_selector(dev))
    sampler.start()
    t_end = time.perf_counter() + 1.5
    while time.perf_counter() < t_end:
        for _ in range(2 if ep else 20):
            run_step()
        torch.cuda.synchronize()

    def timed(fn, n):
        """Sum of per-step device times (CUDA events on the launch stream), with a
        256 MiB write between steps to evict the 126 MB L2; max over ranks."""
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(n):
            flush.zero_()
            starts[i].record()
            fn()
            ends[i].record()
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        tot = sum(a.elapsed_time(b) for a, b in zip(starts, ends))
        t = torch.tensor([tot], device=dev, dtype=torch.float64)
        if ws > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    job_ms = timed(run_step, args.steps)
    clocks = sampler.stop()
    launches = per_step_launches * args.steps
    ms_per_step = job_ms / args.steps
    value = T * ws * args.steps / (job_ms / 1e3)
    eager_ms = timed(lambda: step(x, gout), args.steps) / args.steps

    # per-kernel device time (CUDA events around each of our launches, eager steps)
    with torch.no_grad():
        xf = x.detach().reshape(-1, H)
        lg = layer.router(xf)
        sel = torch.topk(torch.sigmoid(lg.float()), cfg["top_k"], dim=-1).indices
        tpe = torch.bincount(sel.reshape(-1), minlength=layer.num_experts)
        if ep:  # GEMM FLOPs of this rank: rows it receives for its own experts
            dist.all_reduce(tpe)
            mine = torch.zeros_like(tpe)
            mine[layer.local_experts] = 1
            tpe = tpe * mine
        tpe = tpe.cpu().tolist()
    flops = gemm_flops(tpe, cfg)
    reps = 5
    per_kind: dict[str, float] = {}
    kernel_timing = "eager"
    if not ep:
        # the graphed step again, with an event-record node around each of our
        # launches: device time per kernel without host launch overhead
        try:
            tgraph, evs = capture_step(layer, x, gout, kernel_events=True)[::3]
            for _ in range(2):
                tgraph.replay()
            for _ in range(reps):
                flush.zero_()
                tgraph.replay()
                torch.cuda.synchronize()
                for kname, a, b in evs:
                    per_kind[kname] = per_kind.get(kname, 0.0) + a.elapsed_time(b) / reps
            kernel_timing = "graph"
            del tgraph
        except RuntimeError:
            per_kind = {}
    if not per_kind:
        for _ in range(reps):
            flush.zero_()
            with _ops.record_kernel_events() as evs:
                step(x, gout)
            torch.cuda.synchronize()
            for kname, a, b in evs:
                per_kind[kname] = per_kind.get(kname, 0.0) + a.elapsed_time(b) / reps
    gemm_ms = sum(v for k, v in per_kind.items() if k.startswith("grouped_gemm"))
    perm_ms = sum(v for k, v in per_kind.items() if k in ("gather", "weighted_gather", "combine"))
    gemm_names = [kname for kname, _, _ in evs if kname.startswith("grouped_gemm")]
    n_gemm_launches = max(len(gemm_names), 1)
    peak_tf, peak_hbm, peak_kind = measured_peaks()
    achieved = flops / (gemm_ms / 1e3) / 1e12
    traffic_step = ncu_traffic(name)
    roofline = {
        "kernel": f"grouped_gemm_kernel (tcgen05; {n_gemm_launches} launches per step: "
                  f"{', '.join(gemm_names)}; 6 GEMMs)",
        "bound": "tensor",
        "achieved": achieved,
        "peak": peak_tf,
        "unit": "TFLOP/s",
        "frac": achieved / peak_tf,
        "peak_source": f"{peak_kind} bf16 dense (burst)",
        "flops_per_launch": flops / n_gemm_launches,
        "avg_launch_ms": gemm_ms / n_gemm_launches,
        "traffic": (traffic_step / n_gemm_launches) if traffic_step else None,
    }
    pbytes = permute_bytes(cfg)
    permute = {
        "kernels": "gather, combine, weighted gather, unit-weight combine (4 launches per step)",
        "bound": "hbm",
        "achieved": pbytes / (perm_ms / 1e3) / 1e9,
        "peak": peak_hbm,
        "unit": "GB/s",
        "frac": pbytes / (perm_ms / 1e3) / 1e9 / peak_hbm,
        "bytes_per_step": pbytes,
        "ms_per_step": perm_ms,
    }
    kernel_us = {k: round(v * 1e3, 2) for k, v in sorted(per_kind.items())}

    # End to end through the public API with host buffers.  Every step copies its
    # inputs (tokens and output gradient) from pinned host memory and reads its
    # output back to pinned host memory; the copies run on their own streams so
    # step i's upload and step i-1's download overlap step i's compute (two
    # device slots).  The L2 flush still precedes each step's compute.
    if not ep:
        slots = [(x, gout, graph, out_static)]
        x2 = torch.empty_like(x).requires_grad_(True)
        g2 = torch.empty_like(gout)
        with torch.no_grad():
            x2.copy_(x)
            g2.copy_(gout)
        graph2, out2, _, _ = capture_step(layer, x2, g2)
        slots.append((x2, g2, graph2, out2))
    else:
        x2 = x.detach().clone().requires_grad_(True)
        slots = [(x, gout, None, None), (x2, gout.clone(), None, None)]
    out_host = [torch.empty(cfg["batch"], cfg["seq"], H, dtype=torch.bfloat16).pin_memory()
                for _ in range(2)]

    def e2e_run(n):
        comp = torch.cuda.current_stream()
        up, up2, down = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
        ev = lambda: torch.cuda.Event()  # noqa: E731
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        in_ready = [ev() for _ in range(n)]
        computed = [ev() for _ in range(n)]
        fetched = [ev() for _ in range(n)]
        outs = [None] * n
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0.record(comp)

        def upload(i):
            # tokens and output gradient on two copy streams (two DMA engines)
            xs, gs = slots[i % 2][0], slots[i % 2][1]
            for st in (up, up2):
                st.wait_event(t0)
                if i >= 2:
                    st.wait_event(computed[i - 2])  # the slot's previous step is done with it
            with torch.no_grad():
                with torch.cuda.stream(up):
                    xs.copy_(x_host, non_blocking=True)
                with torch.cuda.stream(up2):
                    gs.copy_(g_host, non_blocking=True)
                    gs_done = torch.cuda.Event()
                    gs_done.record(up2)
                up.wait_event(gs_done)
                in_ready[i].record(up)

        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            xs, gs, gr, os_ = slots[i % 2]
            comp.wait_event(in_ready[i])
            if i >= 2:
                comp.wait_event(fetched[i - 2])  # the slot's output was read back
            flush.zero_()
            if gr is not None:
                gr.replay()
                o = os_
            else:
                o = step(xs, gs)
            outs[i] = o
            computed[i].record(comp)
            down.wait_event(computed[i])
            with torch.cuda.stream(down):
                out_host[i % 2].copy_(o.detach(), non_blocking=True)
                fetched[i].record(down)
        comp.wait_event(fetched[n - 1])
        t1.record(comp)
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        t = torch.tensor([t0.elapsed_time(t1)], device=dev, dtype=torch.float64)
        if ws > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    e2e_run(3)
    e2e_ms = e2e_run(args.steps)
    e2e_value = T * ws * args.steps / (e2e_ms / 1e3)
    torch.cuda.synchronize()
    e2e_ok = bool(torch.equal(out_host[(args.steps - 1) % 2],
                              slots[(args.steps - 1) % 2][3].detach().cpu())) if not ep else None
    nbytes = x_host.numel() * 2

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        v, tokens, creps = time_cpu_oracle(cfg)
        cpu = {"value": v, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
               "sample": f"{tokens} of {T} tokens, fwd+bwd, {creps} reps (numpy oracle, bf16 "
                         "rounding points)"}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) random-init weights)",
            "config": {
                "workload": workload_name(name, cfg),
                "global_batch": cfg["batch"] * ws,
                "seq_len": cfg["seq"],
                "parallelism": (f"expert parallel over {ws} GPUs ({layer.num_experts} experts "
                                f"sharded, NCCL all-to-all dispatch/combine), {T} tokens per GPU, "
                                + ("experts placed by the router's measured load over these "
                                   "tokens" if args.placement == "load" else
                                   "round-robin expert placement"))
                if ep else (f"{ws} independent replicas, {T} tokens each, no collective (the "
                            "config's experts fit one GPU; expert parallelism is the c5 "
                            "config)") if ws > 1 else "single GPU",
                "l2": "flushed by a 256 MiB write between timed steps",
            },
            "roofline": roofline,
            "permute_roofline": permute,
            "kernel_us_per_step": kernel_us,
            "kernel_timing": kernel_timing,
            "eager_ms_per_step": eager_ms,
            "execution": ("step captured once in a CUDA graph and replayed (eager time in "
                          "eager_ms_per_step)") if not ep else
                         "eager (expert-parallel exchange sizes are read on the host)",
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": 2 * nbytes,
                    "d2h_bytes_per_step": nbytes, "ms_per_step": e2e_ms / args.steps,
                    "copies": "pinned host -> device on two copy streams (tokens, output "
                              "gradient) and device -> host on a third, overlapped with the "
                              "neighbouring steps' compute (two device slots)",
                    "output_matches_device": e2e_ok},
            "gpu_launches": launches,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c3")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--placement", choices=["load", "round-robin"], default="load",
                    help="expert placement of the expert-parallel config")
    ap.add_argument("--profile-step", action="store_true",
                    help="run the warm-up steps plus one eager step, print nothing (for ncu)")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference(args, cfg, args.config)
    return run_b200(args, cfg, args.config)


if __name__ == "__main__":
    sys.exit(main())
