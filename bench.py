"""Benchmark: MoE layer forward + backward tokens/s on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config c3]

A step is one training pass of the MoE layer over one synthetic batch:
`out, aux, f_i = layer(x); out.backward(g)` (router, routing, gather, grouped
GEMM up with relu^2, grouped GEMM down, weighted combine, and the full
backward).  The default workload (c3) is the 768-hidden variable-expert
layer: n_embd=768, experts 4x512 + 8x256 + 4x128, top-2, batch 8 x seq 1024 =
8192 tokens, bf16, x ~ N(0,1), weights N(0,0.02), router from a random-init
linear.

Execution: the layer never synchronises the host, so the step is captured once
in a CUDA graph and replayed (the eager time is reported beside it).

Timing: W untimed warm-up steps, then exactly K steps, each bracketed by CUDA
events on the launch stream, with a 256 MiB write between steps to flush the
126 MB L2; barrier + synchronize on both sides; the per-rank time is the sum
of the K step times and the job time is the max over ranks.  `value` =
tokens processed by all ranks / job time.  At N > 1 every rank runs its own
c3 layer on its own tokens (weak scaling, no collective: c3's experts fit one
GPU); the expert-parallel config is reported under `ep_c5` at every N.

Extra keys:
  roofline         the grouped-GEMM engine at the headline config: algorithmic
                   FLOPs 12*H*sum_e n_e*w_e per step over the device time of a
                   CUDA graph holding only the step's GEMM launches (same
                   buffers, L2 flushed before each replay), against the
                   measured bf16 peak
  permute_roofline gather / combine kernels against the measured HBM copy
                   bandwidth (algorithmic bytes 4*(T+A)*H*2 + 2*A*2 per step)
  c4               the 2048-hidden 64-expert top-8 layer (N=1): tokens/s, GEMM
                   and permutation rooflines
  route_roofline   routing alone at A = 131072 and 524288 assignments (N=1)
  ep_c5            the 4096-hidden 128-expert top-8 layer with its experts
                   sharded over the N GPUs (dispatch and combine kernels over
                   NVLink peer memory; at N=1 a one-rank group): tokens/s, GEMM roofline,
                   and an in-run parity check of every rank's output and dX
                   against the unsharded layer on a token slice
  cpu_baseline     the reference's own kernels (triton_moe from baseline/_ref)
                   under TRITON_INTERPRET=1 on the host cores, fp32, on a token
                   sample of the workload; cpu_baseline_port: the numpy oracle
  e2e              pinned host input -> device, fwd+bwd, output -> host
  gpu_launches, clocks

`--impl reference` times the reference implementation itself (never this
package): its Triton kernels under TRITON_INTERPRET=1 on the host cores (the
line's value, a bounded token sample per step, steps spread over worker
processes), plus, under `triton_gpu`, the same reference layer compiled by
Triton on the B200 at the full workload.
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
PKG_DIR = ROOT / "triton-variable-moe_b200"
REF_DIR = ROOT / "baseline" / "_ref"  # the reference package (triton_moe), git-ignored

METRIC = "MoE layer fwd+bwd tokens/s"

CONFIGS = {
    "c2u": dict(n_embd=256, expert_sizes=[(8, 512)], top_k=2, batch=8, seq=512, zipf=False),
    "c2v": dict(n_embd=256, expert_sizes=[(4, 512), (4, 256)], top_k=2, batch=8, seq=512, zipf=False),
    "c3": dict(n_embd=768, expert_sizes=[(4, 512), (8, 256), (4, 128)], top_k=2, batch=8, seq=1024,
               zipf=False),
    "c4": dict(n_embd=2048, expert_sizes=[(64, 1024)], top_k=8, batch=1, seq=16384, zipf=True),
    # the expert-parallel config: its experts are sharded over the GPUs
    "c5": dict(n_embd=4096, expert_sizes=[(32, 2048), (64, 1024), (32, 512)], top_k=8, batch=1,
               seq=65536, zipf=True, ep=True),
}

# Tokens per step of the reference's interpreted CPU run (its cost is set by
# the padded tile count, ~50 s per c3 step on one core).
REF_CPU_TOKENS = 256
# DRAM bytes (read + write) of one c3 step's grouped-GEMM launches, summed over
# the launches, from one ncu capture (--metrics dram__bytes_read.sum,
# dram__bytes_write.sum; committed summary profiles/grouped_gemm_c3.md).
NCU_GEMM_DRAM_BYTES_PER_STEP = {"c3": 144706560}


def _pkg_path():
    if str(PKG_DIR) not in sys.path:
        sys.path.insert(0, str(PKG_DIR))
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))


def workload_name(name: str, cfg: dict) -> str:
    sizes = "+".join(f"{c}x{w}" for c, w in cfg["expert_sizes"])
    return (f"{name}: MoE layer n_embd={cfg['n_embd']} experts {sizes} top-{cfg['top_k']} "
            f"tokens={cfg['batch'] * cfg['seq']}" + (" zipf(1.1) router bias" if cfg["zipf"] else ""))


def config_dict(name: str, cfg: dict, ws: int) -> dict:
    """The `config` of the JSON line (the same for both arms)."""
    return {
        "workload": workload_name(name, cfg),
        "global_batch": cfg["batch"] * ws,
        "seq_len": cfg["seq"],
        "parallelism": (f"{ws} independent replicas, {cfg['batch'] * cfg['seq']} tokens each, no "
                        "collective (the config's experts fit one GPU; expert parallelism is "
                        "ep_c5)") if ws > 1 else "single GPU",
        "l2": "flushed by a 256 MiB write between timed steps",
    }


def widths_of(cfg):
    return [w for c, w in cfg["expert_sizes"] for _ in range(c)]


def gemm_flops(tokens_per_expert, cfg) -> float:
    """12 * H * sum_e n_e * w_e: the six GEMMs of fwd+bwd, unpadded counts."""
    H = cfg["n_embd"]
    return float(sum(12 * H * int(n) * w for n, w in zip(tokens_per_expert, widths_of(cfg))))


def permute_bytes(cfg, tokens=None) -> float:
    """Unique bytes moved by gather + scatter forward and their backward mirrors."""
    T = tokens if tokens is not None else cfg["batch"] * cfg["seq"]
    A = T * cfg["top_k"]
    H = cfg["n_embd"]
    return float(4 * (T + A) * H * 2 + 2 * A * 2)


def route_bytes(A: int, P: int, id_bytes: int = 4) -> float:
    """Routing's compulsory bytes: the expert ids read once; bin_ids, indices and
    the two row maps (assignment -> padded row, padded row -> assignment) written."""
    return float(A * id_bytes + 4 * A + 4 * A + 4 * A + 4 * P)


def zipf_bias(E, seed, s=1.1):
    import torch

    g = torch.Generator().manual_seed(seed)
    ranks = torch.randperm(E, generator=g).float() + 1.0
    logp = -s * torch.log(ranks)
    logp = logp - torch.logsumexp(logp, 0)
    return logp - logp.mean()


def init_weights(layer, cfg, seed: int, device):
    """The workload's weights, identical for both arms on one device type: after
    construction, seed, then router.weight, w1, w2 ~ N(0, 0.02) in that order;
    with the Zipf bias the router becomes an nn.Linear with that bias."""
    import torch

    torch.manual_seed(seed)
    with torch.no_grad():
        layer.router.weight.normal_(0, 0.02)
        layer.w1.normal_(0, 0.02)
        layer.w2.normal_(0, 0.02)
    if cfg["zipf"]:
        r = torch.nn.Linear(cfg["n_embd"], layer.num_experts, bias=True, device=device)
        with torch.no_grad():
            r.weight.copy_(layer.router.weight)
            r.bias.copy_(zipf_bias(layer.num_experts, seed + 1).to(device))
        layer.router = r
    return layer


def build_layer(cfg, device, seed=0):
    """This package's layer (bf16), built directly on `device`."""
    import torch

    _pkg_path()
    from moe_b200 import TritonMoEConfig, TritonMoEMLP

    with torch.device(device):
        layer = TritonMoEMLP(TritonMoEConfig(n_embd=cfg["n_embd"], expert_sizes=cfg["expert_sizes"],
                                             num_active_experts=cfg["top_k"], block_size=64))
    init_weights(layer, cfg, seed, device)
    return layer.to(device=device, dtype=torch.bfloat16)


def make_tokens(cfg, rank: int, tokens=None):
    """(x, output gradient) of the workload for `rank`: bf16 N(0,1), seeded."""
    import torch

    T = tokens if tokens is not None else cfg["batch"] * cfg["seq"]
    g = torch.Generator(device="cpu").manual_seed(1234 + rank)
    shape = (cfg["batch"], cfg["seq"], cfg["n_embd"]) if tokens is None else (1, T, cfg["n_embd"])
    x = torch.randn(*shape, generator=g).to(torch.bfloat16)
    gout = torch.randn(*shape, generator=g).to(torch.bfloat16)
    return x, gout


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


def time_cpu_port(cfg, tokens: int, seed=0, budget_s=10.0):
    """The numpy oracle (a restatement of the reference, bf16 rounding points) on
    a `tokens`-token sample of the workload: tokens/s."""
    import numpy as np
    import torch

    torch.manual_seed(seed)
    g = torch.Generator().manual_seed(seed + 7)
    H, E, k = cfg["n_embd"], sum(c for c, _ in cfg["expert_sizes"]), cfg["top_k"]
    x = torch.randn(tokens, H, generator=g)
    wr = torch.randn(E, H, generator=g) * 0.02
    w1 = (torch.randn(H, sum(widths_of(cfg)), generator=g) * 0.02).numpy()
    w2 = (torch.randn(sum(widths_of(cfg)), H, generator=g) * 0.02).numpy()
    probs = torch.sigmoid(x @ wr.T)
    w, sel = torch.topk(probs, k, dim=-1)
    w = w / (w.sum(-1, keepdim=True) + 1e-20)
    gout = torch.randn(tokens, H, generator=g).numpy()
    args = (x.numpy(), w1, w2, sel.reshape(-1).numpy().astype(np.int64), w.reshape(-1).numpy(), gout)
    t0 = time.perf_counter()
    cpu_oracle_step(cfg, *args)
    first = time.perf_counter() - t0
    reps = max(1, min(20, int(budget_s / max(first, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(reps):
        cpu_oracle_step(cfg, *args)
    return tokens * reps / (time.perf_counter() - t0), reps


# ------------------------------------------------------------------ the reference
def load_reference(interpret: bool):
    """Import the reference package triton_moe from baseline/_ref.  Under the
    Triton interpreter two harness-only adjustments are made in memory (the
    reference files are untouched): fused_route's `selected_experts.is_cuda`
    assert (fused_cumsum.py:119) is dropped by re-executing the function's
    source without that line, and each autotuned GEMM kernel is pinned to one
    of its own configs (BLOCK_M = BLOCK_N = 128, BLOCK_K = 64;
    grouped_gemm.py:36-72), because autotuning needs a GPU."""
    if interpret:
        os.environ["TRITON_INTERPRET"] = "1"
    if not (REF_DIR / "triton_moe").is_dir():
        raise RuntimeError(f"reference package not installed under {REF_DIR}")
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import triton_moe.moe as moe_mod

    if interpret:
        import inspect

        import triton_moe.kernels as K
        import triton_moe.kernels.fused_cumsum as fc
        import triton_moe.kernels.grouped_gemm as gg

        src = inspect.getsource(fc.fused_route)
        src = "\n".join(ln for ln in src.splitlines()
                        if "is_cuda" not in ln and not ln.lstrip().startswith("@"))
        ns = dict(vars(fc))
        exec(src, ns)
        fc.fused_route = moe_mod.fused_route = K.fused_route = ns["fused_route"]
        for name in dir(gg):
            k = getattr(gg, name)
            if hasattr(k, "configs") and name.startswith("_grouped"):
                big = [c for c in k.configs if c.kwargs.get("BLOCK_M") == 128
                       and c.kwargs.get("BLOCK_N") == 128 and c.kwargs.get("BLOCK_K") == 64]
                k.configs = [big[0] if big else k.configs[0]]
    return moe_mod


def build_ref_layer(moe_mod, cfg, device, seed=0):
    import torch

    with torch.device(device):
        layer = moe_mod.TritonMoEMLP(moe_mod.TritonMoEConfig(
            n_embd=cfg["n_embd"], expert_sizes=cfg["expert_sizes"],
            num_active_experts=cfg["top_k"], block_size=64))
    return init_weights(layer, cfg, seed, device)


_REF_STATE: dict = {}


def _ref_worker_init(cfg_name: str, tokens: int):
    """Worker process of the interpreted reference: one core, fp32 (the
    interpreter's bf16 dot is unusable in this Triton version)."""
    import torch

    torch.set_num_threads(1)
    moe_mod = load_reference(interpret=True)
    cfg = CONFIGS[cfg_name]
    layer = build_ref_layer(moe_mod, cfg, "cpu").float()
    x, gout = make_tokens(cfg, 0, tokens)
    _REF_STATE.update(layer=layer, x=x.float(), g=gout.float())


def _ref_worker_step(_i: int) -> float:
    """One forward + backward of the reference layer on the sample; seconds."""
    layer, x, g = _REF_STATE["layer"], _REF_STATE["x"], _REF_STATE["g"]
    t0 = time.perf_counter()
    xi = x.clone().requires_grad_(True)
    layer.zero_grad(set_to_none=True)
    out, _aux, _f = layer(xi)
    out.backward(g)
    return time.perf_counter() - t0


def time_reference_cpu(cfg_name: str, tokens: int, warmup: int, steps: int, procs: int) -> dict:
    """The reference's kernels under TRITON_INTERPRET=1 on the host cores: the
    steps run as tasks over `procs` single-threaded worker processes; the
    timed region is the wall time of the K timed steps (after the warm-up
    steps).  Returns tokens/s and the sample description."""
    import concurrent.futures as cf
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    with cf.ProcessPoolExecutor(max_workers=procs, mp_context=ctx, initializer=_ref_worker_init,
                                initargs=(cfg_name, tokens)) as ex:
        if warmup > 0:
            list(ex.map(_ref_worker_step, range(warmup)))
        t0 = time.perf_counter()
        per = list(ex.map(_ref_worker_step, range(steps)))
        wall = time.perf_counter() - t0
    return {"value": tokens * steps / wall, "wall_s": wall, "step_s_median": statistics.median(per),
            "procs": procs}


def ref_gpu_child(args) -> int:
    """(subprocess) The reference layer compiled by Triton on the B200 at the full
    workload, bf16, eager (its forward reads sizes on the host): W warm-up
    steps, K timed steps with CUDA events, L2 flushed between steps."""
    import torch

    moe_mod = load_reference(interpret=False)
    cfg = CONFIGS[args.config]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    layer = build_ref_layer(moe_mod, cfg, dev).to(torch.bfloat16)
    x_h, g_h = make_tokens(cfg, 0)
    x = x_h.to(dev).requires_grad_(True)
    gout = g_h.to(dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def step():
        layer.zero_grad(set_to_none=True)
        x.grad = None
        out, _aux, _f = layer(x)
        out.backward(gout)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        torch.cuda.synchronize()
        tot += a.elapsed_time(b)
    T = cfg["batch"] * cfg["seq"]
    print(json.dumps({"value": T * args.steps / (tot / 1e3), "unit": "tokens/s",
                      "ms_per_step": tot / args.steps, "dtype": "bf16",
                      "what": "the reference's TritonMoEMLP (Triton kernels compiled for this "
                              "GPU) at the full workload, eager"}), flush=True)
    return 0


def run_reference(args, cfg, name):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    if not (REF_DIR / "triton_moe").is_dir():
        print(json.dumps({"impl": "reference", "unavailable": f"reference not installed under {REF_DIR}"}))
        return 0
    T = cfg["batch"] * cfg["seq"]
    tokens = min(T, REF_CPU_TOKENS)
    # the reference on the GPU first (its own subprocess: no interpreter there)
    gpu = None
    try:
        r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                            "--ref-gpu-child", "--config", name, "--steps", str(args.steps),
                            "--warmup", str(args.warmup)], capture_output=True, text=True,
                           timeout=900, env={k: v for k, v in os.environ.items()
                                             if k not in ("TRITON_INTERPRET", "WORLD_SIZE", "RANK",
                                                          "LOCAL_RANK")})
        lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
        gpu = json.loads(lines[-1]) if (r.returncode == 0 and lines) else {
            "unavailable": (r.stderr.strip().splitlines() or ["no output"])[-1][:300]}
    except (subprocess.TimeoutExpired, OSError) as e:
        gpu = {"unavailable": str(e)[:300]}
    # one process per timed step, up to twice the cores: the timed steps run as one wave
    procs = max(1, min(2 * (os.cpu_count() or 1), args.steps))
    cpu = time_reference_cpu(name, tokens, args.warmup, args.steps, procs)
    value = cpu["value"]
    sample = (f"{tokens} of the workload's {T} tokens per step: the reference's TritonMoEMLP "
              f"fwd+bwd (its Triton kernels under TRITON_INTERPRET=1, fp32, GEMMs pinned to "
              f"their 128x128x64 autotune config), {args.steps} timed steps over {procs} "
              f"single-threaded worker processes (median step {cpu['step_s_median']:.1f} s)")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": cpu["wall_s"] / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) random-init weights)",
        "config": config_dict(name, cfg, ws),
        "execution": "host cores (the reference's Triton kernels under the Triton interpreter)",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": min(procs, os.cpu_count() or 1), "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "triton_gpu": gpu,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our arm
def capture_step(layer, x, gout, kernel_events=False, before_capture=None):
    """Capture one fwd+bwd of the layer in a CUDA graph (the layer never
    synchronises the host, so the whole step is capturable).  Returns the graph,
    its static output, how many of our kernels one replay launches and (with
    kernel_events) the (name, start, end) event pairs recorded around each of
    our launches inside the graph.  before_capture: called after the warm-up
    steps, right before the capture."""
    import torch

    from moe_b200.kernels import _ops

    # warm-up and capture on the caller's (non-default) stream: the autograd
    # nodes that accumulate into the long-lived leaves (x, the parameters) then
    # always run on the stream they were created on
    for _ in range(3):
        layer.zero_grad(set_to_none=True)
        x.grad = None
        out, _, _ = layer(x)
        out.backward(gout)
    torch.cuda.synchronize()
    layer.zero_grad(set_to_none=True)
    x.grad = None
    if before_capture is not None:
        before_capture()
    graph = torch.cuda.CUDAGraph()
    l0 = _ops.launch_count
    evs: list = []
    with torch.cuda.graph(graph, stream=torch.cuda.current_stream()):
        if kernel_events:
            with _ops.record_kernel_events(external=True) as evs:
                out, _, _ = layer(x)
                out.backward(gout)
        else:
            out, _, _ = layer(x)
            out.backward(gout)
    return graph, out, _ops.launch_count - l0, evs


GEMM_ENTRY_POINTS = ("moe_grouped_gemm_up_down", "moe_grouped_gemm_down_backward",
                     "moe_grouped_gemm_up_backward")


PERMUTE_ENTRY_POINTS = ("moe_padded_gather", "moe_padded_scatter")


def capture_with_part_graphs(layer, x, gout):
    """capture_step, plus one CUDA graph per group of launches (the step's
    grouped-GEMM launches; its gather / combine launches), each holding those
    launches with the same arguments (the same buffers of the first graph's
    memory pool), so that they can be timed back to back without the
    event-record nodes that break programmatic dependent launch.  Replaying a
    part graph after the step graph rewrites the same values."""
    import torch

    from moe_b200 import _lib

    groups = {"gemm": GEMM_ENTRY_POINTS, "permute": PERMUTE_ENTRY_POINTS}
    names = [n for g in groups.values() for n in g]
    orig = {n: getattr(_lib.lib, n) for n in names}
    calls: list = []

    def wrap(n):
        f = orig[n]

        def call(*a):
            calls.append((n, a))
            return f(*a)

        return call

    for n in names:
        setattr(_lib.lib, n, wrap(n))
    try:
        graph, out, launches, _ = capture_step(layer, x, gout, before_capture=calls.clear)
    finally:
        for n in names:
            setattr(_lib.lib, n, orig[n])
    parts = {}
    for key, entry in groups.items():
        step_calls = [(n, a) for n, a in calls if n in entry]  # the captured step's launches
        gg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gg, stream=torch.cuda.current_stream()):
            st = torch.cuda.current_stream().cuda_stream
            for n, a in step_calls:
                rc = orig[n](*a[:-1], st)  # the stream is every entry point's last argument
                if rc != 0:
                    raise RuntimeError(f"{n} failed in the {key}-only graph: {rc}")
        parts[key] = (gg, [n for n, _ in step_calls])
    return graph, out, launches, parts


def timed_replays(fn, n, flush, ws=1, dist=None, dev=None) -> float:
    """Sum of per-call device times (CUDA events on the launch stream), with a
    256 MiB write before each call to evict the 126 MB L2; max over ranks."""
    import torch

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
    if ws > 1:
        t = torch.tensor([tot], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tot = float(t.item())
    return tot


def routed_counts(layer, x, top_k):
    """Per-expert token counts the layer's router gives x (unpadded)."""
    import torch

    with torch.no_grad():
        xf = x.detach().reshape(-1, x.shape[-1])
        lg = layer.router(xf)
        sel = torch.topk(torch.sigmoid(lg.float()), top_k, dim=-1).indices
        return torch.bincount(sel.reshape(-1), minlength=layer.num_experts)


def kernel_times(layer, x, gout, flush, reps=5):
    """Device time per kernel kind of one step, from a graph of the step with an
    event-record node around each of our launches (the nodes break
    programmatic dependent launch, so these are upper bounds)."""
    tgraph, evs = capture_step(layer, x, gout, kernel_events=True)[::3]
    for _ in range(2):
        tgraph.replay()
    per_kind: dict[str, float] = {}
    import torch

    for _ in range(reps):
        flush.zero_()
        tgraph.replay()
        torch.cuda.synchronize()
        for kname, a, b in evs:
            per_kind[kname] = per_kind.get(kname, 0.0) + a.elapsed_time(b) / reps
    return per_kind


def gemm_roofline(flops, gemm_ms, n_launches, names, peak_tf, peak_kind, traffic_step=None,
                  how=""):
    achieved = flops / (gemm_ms / 1e3) / 1e12
    return {
        "kernel": f"grouped_gemm_kernel (tcgen05; {n_launches} launches per step: "
                  f"{', '.join(names)}; 6 GEMMs)",
        "bound": "tensor",
        "achieved": achieved,
        "peak": peak_tf,
        "unit": "TFLOP/s",
        "frac": achieved / peak_tf,
        "peak_source": f"{peak_kind} bf16 dense (burst)",
        "flops_per_launch": flops / n_launches,
        "avg_launch_ms": gemm_ms / n_launches,
        "gemm_ms_per_step": gemm_ms,
        "timing": how,
        "traffic": (traffic_step / n_launches) if traffic_step else None,
        "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the step's GEMM "
                           "launches (one capture, per launch)") if traffic_step else None,
    }


def permute_roofline(pbytes, perm_ms, peak_hbm):
    return {
        "kernels": "gather, combine, weighted gather, unit-weight combine (4 launches per step)",
        "bound": "hbm",
        "achieved": pbytes / (perm_ms / 1e3) / 1e9,
        "peak": peak_hbm,
        "unit": "GB/s",
        "frac": pbytes / (perm_ms / 1e3) / 1e9 / peak_hbm,
        "bytes_per_step": pbytes,
        "ms_per_step": perm_ms,
    }


def measure_single(name, cfg, dev, flush, steps, warmup, peaks):
    """A single-GPU config (c4) at its full size: graphed step tokens/s, the GEMM
    roofline from a GEMM-only graph, the permutation roofline from a graph of the
    gather / combine launches only."""
    import torch

    layer = build_layer(cfg, dev)
    x_h, g_h = make_tokens(cfg, 0)
    x = x_h.to(dev).requires_grad_(True)
    gout = g_h.to(dev)
    graph, _out, _l, parts = capture_with_part_graphs(layer, x, gout)
    gg, names = parts["gemm"]
    pg, _pnames = parts["permute"]
    for _ in range(max(warmup, 3)):
        graph.replay()
        gg.replay()
        pg.replay()
    step_ms = timed_replays(graph.replay, steps, flush) / steps
    gemm_ms = timed_replays(gg.replay, steps, flush) / steps
    perm_ms = timed_replays(pg.replay, steps, flush) / steps
    per_kind = kernel_times(layer, x, gout, flush)
    T = cfg["batch"] * cfg["seq"]
    flops = gemm_flops(routed_counts(layer, x, cfg["top_k"]).cpu().tolist(), cfg)
    out = {
        "workload": workload_name(name, cfg),
        "value": T / (step_ms / 1e3),
        "unit": "tokens/s",
        "ms_per_step": step_ms,
        "roofline": gemm_roofline(flops, gemm_ms, len(names), names, peaks[0], peaks[2],
                                  how="CUDA graph of the step's GEMM launches only, L2 flushed "
                                      "before each replay"),
        "permute_roofline": dict(
            permute_roofline(permute_bytes(cfg), perm_ms, peaks[1]),
            timing="CUDA graph of the step's gather / combine launches only, L2 flushed "
                   "before each replay"),
        "kernel_us_per_step": {k: round(v * 1e3, 2) for k, v in sorted(per_kind.items())},
    }
    del graph, gg, pg, layer
    torch.cuda.empty_cache()
    return out


def measure_route(dev, flush, steps, peaks):
    """Routing alone (moe_route) at the c4 and c5 assignment counts: graph of one
    routing call on skewed int32 ids, L2 flushed before each replay."""
    import torch

    from moe_b200.kernels import _ops

    res = {}
    for A, E in ((131072, 64), (524288, 128)):
        g = torch.Generator(device="cpu").manual_seed(A)
        p = 1.0 / torch.arange(1, E + 1, dtype=torch.float64) ** 1.1
        sel = torch.multinomial(p / p.sum(), A, replacement=True, generator=g).to(torch.int32).to(dev)
        r = _ops.route(sel, E, 64)
        torch.cuda.synchronize()
        P = int(r.expert_token_offsets[-1].item())
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=torch.cuda.current_stream()):
            _ops.route(sel, E, 64)
        for _ in range(3):
            gr.replay()
        ms = timed_replays(gr.replay, steps, flush) / steps
        b = route_bytes(A, P)
        res[f"A={A},E={E}"] = {"ms": ms, "bytes": b, "achieved": b / (ms / 1e3) / 1e9,
                                "unit": "GB/s", "frac": b / (ms / 1e3) / 1e9 / peaks[1],
                                "launches": 2}
    return res


def run_ep_c5(args, dev, ws, rank, flush, peaks):
    """The expert-parallel config at this N: experts sharded over the ranks of
    the default group (N=1: a one-rank group, so the same exchange code path
    runs), every rank with its own 65536 tokens.  Timed eagerly (the exchange
    plan is built on the host from the all-gathered counts once per forward).
    Parity: on a token slice every rank compares the sharded layer's output
    and dX with the unsharded layer (same weights, on this GPU)."""
    import torch
    import torch.distributed as dist

    from moe_b200.kernels import _ops

    cfg = CONFIGS["c5"]
    T, H = cfg["batch"] * cfg["seq"], cfg["n_embd"]
    full = build_layer(cfg, dev)
    x_h, g_h = make_tokens(cfg, rank)
    x = x_h.to(dev)
    layer = build_ep_layer(cfg, dev, full, calib_x=x if args.placement == "load" else None)

    # parity on a slice
    S = 2048
    xs = x[:, :S].clone().requires_grad_(True)
    gs = g_h[:, :S].to(dev)
    out_ep, _, _ = layer(xs)
    out_ep.backward(gs)
    xf = xs.detach().clone().requires_grad_(True)
    out_full, _, _ = full(xf)
    out_full.backward(gs)
    torch.cuda.synchronize()

    def err(a, b):
        a, b = a.float(), b.float()
        bad = ((a - b).abs() > 1e-2 * b.abs().max() + 2e-2 * b.abs()).sum().item()
        return float((a - b).abs().max().item()), int(bad)

    e_out, bad_out = err(out_ep.detach(), out_full.detach())
    e_dx, bad_dx = err(xs.grad, xf.grad)
    ok = torch.tensor([1 if (bad_out == 0 and bad_dx == 0) else 0], device=dev)
    if ws > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    parity = {"ok": bool(ok.item()), "tokens_per_rank": S, "max_abs_err_out": e_out,
              "max_abs_err_dx": e_dx, "bit_exact_rank0": e_out == 0.0 and e_dx == 0.0,
              "tolerance": "|a-b| <= 1e-2 max|b| + 2e-2 |b| (bf16 vs the unsharded layer)"}
    del out_ep, out_full, xs, xf, full
    torch.cuda.empty_cache()

    xr = x.requires_grad_(True)
    gout = g_h.to(dev)

    def step():
        layer.zero_grad(set_to_none=True)
        xr.grad = None
        out, _aux, _f = layer(xr)
        out.backward(gout)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 20))
    job_ms = timed_replays(step, steps, flush, ws, dist, dev)
    ms = job_ms / steps
    # per-kernel device times of one eager step on this rank
    reps = 2
    per_kind: dict[str, float] = {}
    for _ in range(reps):
        flush.zero_()
        with _ops.record_kernel_events() as evs:
            step()
        torch.cuda.synchronize()
        for kname, a, b in evs:
            per_kind[kname] = per_kind.get(kname, 0.0) + a.elapsed_time(b) / reps
    tpe = routed_counts(layer, xr, cfg["top_k"])
    if ws > 1:
        dist.all_reduce(tpe)
    mine = torch.zeros_like(tpe)
    mine[layer.local_experts] = 1
    flops = gemm_flops((tpe * mine).cpu().tolist(), cfg)
    gemm_ms = sum(v for k, v in per_kind.items() if k.startswith("grouped_gemm"))
    gflops = torch.tensor([flops / (gemm_ms / 1e3) / 1e12], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(gflops, op=dist.ReduceOp.MIN)
    names = sorted({k for k in per_kind if k.startswith("grouped_gemm")})
    res = {
        "workload": workload_name("c5", cfg) + " per GPU",
        "value": T * ws * steps / (job_ms / 1e3),
        "unit": "tokens/s",
        "ms_per_step": ms,
        "n_gpus": ws,
        "steps": steps,
        "parallelism": (f"experts sharded over {ws} GPU(s) ({'placed by measured router load' if args.placement == 'load' else 'round-robin'}), "
                        f"dispatch/combine over NVLink peer memory (NCCL barriers), {T} tokens per GPU"),
        "parity": parity,
        "roofline": {"bound": "tensor", "unit": "TFLOP/s", "peak": peaks[0],
                     "achieved_min_over_ranks": float(gflops.item()),
                     "frac": float(gflops.item()) / peaks[0],
                     "timing": "event-timed grouped-GEMM launches of one eager step, this rank's "
                               "FLOPs; slowest rank"},
        "kernel_ms_per_step_rank0": {k: round(v, 3) for k, v in sorted(per_kind.items())},
        "exchange": ("fused dispatch (gather + NVLink push into the owners' layouts) and "
                     "combine (NVLink pull + weighted sum) kernels on an exchange stream, "
                     "token chunks pipelined against the grouped GEMMs, NCCL barriers"),
    }
    perm_ms = sum(v for k, v in per_kind.items() if k in ("ep_dispatch", "ep_combine"))
    if ws == 1 and perm_ms > 0:
        # at one rank the fused exchange kernels move the same bytes as the
        # single-GPU gather / combine kernels, all through local HBM
        res["permute_roofline"] = permute_roofline(permute_bytes(cfg), perm_ms, peaks[1])
        res["permute_roofline"]["kernels"] = ("ep_dispatch (gather fused with the push) and "
                                              "ep_combine (pull fused with the weighted sum), "
                                              "forward and backward")
    del layer
    torch.cuda.empty_cache()
    return res


def build_ep_layer(cfg, device, full, calib_x=None):
    """The layer `full` (same weights) with its experts sharded over the ranks of
    the default process group.  With calib_x (this rank's tokens), the experts
    are placed by the load the router gives them over all ranks' tokens;
    else round-robin."""
    import torch

    from moe_b200 import TritonMoEConfig
    from moe_b200.ep import ExpertParallelMoEMLP, measure_expert_loads

    mcfg = TritonMoEConfig(n_embd=cfg["n_embd"], expert_sizes=cfg["expert_sizes"],
                           num_active_experts=cfg["top_k"], block_size=64)
    loads = measure_expert_loads(full.router, calib_x, cfg["top_k"]) if calib_x is not None else None
    with torch.device(device):
        layer = ExpertParallelMoEMLP(mcfg, expert_loads=loads)
    if cfg["zipf"]:
        import copy

        layer.router = copy.deepcopy(full.router)
    layer.load_full_state_dict({k: v for k, v in full.state_dict().items()})
    return layer.to(device=device, dtype=torch.bfloat16)


def run_b200(args, cfg, name):
    import datetime

    import torch
    import torch.distributed as dist

    _pkg_path()
    from moe_b200.kernels import _ops

    ws, rank, local = dist_env()
    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "error": "no CUDA device"}))
        return 1
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # every step (eager, captured, replayed) runs on one non-default stream
    torch.cuda.set_stream(torch.cuda.Stream(device=dev))
    timeout = datetime.timedelta(minutes=10)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timeout)
    else:
        # a one-rank group, so that ep_c5 runs its exchange code path at N=1 too
        dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                                device_id=dev, timeout=timeout)

    T = cfg["batch"] * cfg["seq"]
    H = cfg["n_embd"]
    peaks = measured_peaks()
    x_host, g_host = make_tokens(cfg, rank)
    x_host, g_host = x_host.pin_memory(), g_host.pin_memory()
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
        dist.destroy_process_group()
        return 0

    graph, out_static, per_step_launches, parts = capture_with_part_graphs(layer, x, gout)
    gemm_graph, gemm_names = parts["gemm"]
    perm_graph, perm_names = parts["permute"]
    for _ in range(3):
        graph.replay()
        gemm_graph.replay()
        perm_graph.replay()
    torch.cuda.synchronize()

    # clock samples: a ~1.5 s soak of the same step right before the timed loop
    sampler = ClockSampler(gpu_selector(dev))
    sampler.start()
    t_end = time.perf_counter() + 1.5
    while time.perf_counter() < t_end:
        for _ in range(20):
            graph.replay()
        torch.cuda.synchronize()

    job_ms = timed_replays(graph.replay, args.steps, flush, ws, dist, dev)
    clocks = sampler.stop()
    launches = per_step_launches * args.steps
    ms_per_step = job_ms / args.steps
    value = T * ws * args.steps / (job_ms / 1e3)
    eager_ms = timed_replays(lambda: step(x, gout), args.steps, flush, ws, dist, dev) / args.steps
    # the GEMM launches alone, back to back (programmatic dependent launch intact)
    gemm_ms = timed_replays(gemm_graph.replay, args.steps, flush) / args.steps
    flops = gemm_flops(routed_counts(layer, x, cfg["top_k"]).cpu().tolist(), cfg)
    roofline = gemm_roofline(flops, gemm_ms, len(gemm_names), gemm_names, peaks[0], peaks[2],
                             traffic_step=NCU_GEMM_DRAM_BYTES_PER_STEP.get(name),
                             how="CUDA graph of the step's GEMM launches only (same buffers), "
                                 "L2 flushed before each replay")
    per_kind = kernel_times(layer, x, gout, flush)
    # the gather / combine launches alone, back to back (as for the GEMMs)
    perm_ms = timed_replays(perm_graph.replay, args.steps, flush) / args.steps
    permute = permute_roofline(permute_bytes(cfg), perm_ms, peaks[1])
    permute["kernels"] += f" ({', '.join(perm_names)})"
    permute["timing"] = ("CUDA graph of the step's gather / combine launches only (same "
                         "buffers), L2 flushed before each replay")
    permute["ms_per_step_event_timed"] = sum(
        v for k, v in per_kind.items() if k in ("gather", "weighted_gather", "combine"))
    kernel_us = {k: round(v * 1e3, 2) for k, v in sorted(per_kind.items())}

    # End to end through the public API with host buffers.  Every step copies its
    # inputs (tokens and output gradient) from pinned host memory and reads its
    # output back to pinned host memory; the copies run on their own streams so
    # step i's upload and step i-1's download overlap step i's compute (two
    # device slots).  The L2 flush still precedes each step's compute.
    slots = [(x, gout, graph, out_static)]
    x2 = torch.empty_like(x).requires_grad_(True)
    g2 = torch.empty_like(gout)
    with torch.no_grad():
        x2.copy_(x)
        g2.copy_(gout)
    graph2, out2, _, _ = capture_step(layer, x2, g2)
    slots.append((x2, g2, graph2, out2))
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
            _xs, _gs, gr, os_ = slots[i % 2]
            comp.wait_event(in_ready[i])
            if i >= 2:
                comp.wait_event(fetched[i - 2])  # the slot's output was read back
            flush.zero_()
            gr.replay()
            computed[i].record(comp)
            down.wait_event(computed[i])
            with torch.cuda.stream(down):
                out_host[i % 2].copy_(os_.detach(), non_blocking=True)
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
                              slots[(args.steps - 1) % 2][3].detach().cpu()))
    nbytes = x_host.numel() * 2
    del slots, graph, graph2, gemm_graph, perm_graph, layer, out_static, out2, x, x2, gout, g2
    torch.cuda.empty_cache()

    extra = {}
    if ws == 1 and not args.no_extras:
        extra["c4"] = measure_single("c4", CONFIGS["c4"], dev, flush, min(args.steps, 20),
                                     args.warmup, peaks)
        extra["route_roofline"] = measure_route(dev, flush, min(args.steps, 50), peaks)
    if not args.no_extras:
        extra["ep_c5"] = run_ep_c5(args, dev, ws, rank, flush, peaks)

    cpu = port = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        _pkg_path()
        pv, preps = time_cpu_port(cfg, min(T, REF_CPU_TOKENS))
        port = {"value": pv, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
                "sample": f"{min(T, REF_CPU_TOKENS)} of {T} tokens, fwd+bwd, {preps} reps (numpy "
                          "oracle, bf16 rounding points)"}
        if (REF_DIR / "triton_moe").is_dir():
            procs = max(1, min(os.cpu_count() or 1, 16))
            try:
                r = time_reference_cpu(name, min(T, REF_CPU_TOKENS), 0, procs, procs)
                cpu = {"value": r["value"], "unit": "tokens/s", "cores": procs,
                       "kind": "reference",
                       "sample": f"{min(T, REF_CPU_TOKENS)} of {T} tokens per step: the "
                                 "reference's TritonMoEMLP fwd+bwd under TRITON_INTERPRET=1 "
                                 f"(fp32), one step on each of {procs} single-threaded worker "
                                 f"processes in parallel (median step {r['step_s_median']:.1f} s)"}
            except Exception as e:  # noqa: BLE001 - reported, the port stays
                cpu = dict(port, note=f"reference run failed: {str(e)[:200]}")
        else:
            cpu = port

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
            "config": config_dict(name, cfg, ws),
            "roofline": roofline,
            "permute_roofline": permute,
            "kernel_us_per_step": kernel_us,
            "kernel_timing": ("graph of the step with an event-record node around each of our "
                              "launches (upper bounds: the nodes break programmatic dependent "
                              "launch)"),
            "eager_ms_per_step": eager_ms,
            "execution": "step captured once in a CUDA graph and replayed (eager time in "
                         "eager_ms_per_step)",
            "cpu_baseline": cpu,
            "cpu_baseline_port": port,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": 2 * nbytes,
                    "d2h_bytes_per_step": nbytes, "ms_per_step": e2e_ms / args.steps,
                    "copies": "pinned host -> device on two copy streams (tokens, output "
                              "gradient) and device -> host on a third, overlapped with the "
                              "neighbouring steps' compute (two device slots)",
                    "output_matches_device": e2e_ok},
            "gpu_launches": launches,
            "clocks": clocks,
            **extra,
        }
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c3")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the c4, route and ep_c5 measurements")
    ap.add_argument("--placement", choices=["load", "round-robin"], default="load",
                    help="expert placement of the expert-parallel config")
    ap.add_argument("--profile-step", action="store_true",
                    help="run the warm-up steps plus one eager step, print nothing (for ncu)")
    ap.add_argument("--ref-gpu-child", action="store_true", help=argparse.SUPPRESS)
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        if args.ref_gpu_child:
            return ref_gpu_child(args)
        return run_reference(args, cfg, args.config)
    return run_b200(args, cfg, args.config)


if __name__ == "__main__":
    sys.exit(main())
