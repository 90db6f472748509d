"""Generate golden vectors by running the REFERENCE implementation on CPU.

The reference package (hbfreed/triton-variable-moe, `triton_moe`) is Triton
code.  Here it runs unmodified on CPU under TRITON_INTERPRET=1, in fp32 (the
interpreter's bf16 dot is unusable in this Triton version).  Two harness-only
adjustments are made in memory, never to the reference files:
  1. fused_route asserts `selected_experts.is_cuda` (fused_cumsum.py:119); the
     function source is re-executed without that one line;
  2. each @triton.autotune kernel is pinned to its first config, because
     autotuning needs a GPU driver.

Usage (needs the reference checkout; the outputs are committed):
    python tests/golden/make_golden.py --ref /path/to/reference

Outputs: tests/golden/*.npz (small; inputs and reference outputs).
"""

from __future__ import annotations

import argparse
import inspect
import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def load_reference(ref: str):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref)
    import triton_moe.kernels.fused_cumsum as fc
    import triton_moe.kernels.grouped_gemm as gg
    import triton_moe.moe as moe_mod

    src = inspect.getsource(fc.fused_route)
    src = "\n".join(
        ln for ln in src.splitlines() if "is_cuda" not in ln and not ln.lstrip().startswith("@")
    )
    ns = dict(vars(fc))
    exec(src, ns)
    fc.fused_route = ns["fused_route"]
    moe_mod.fused_route = ns["fused_route"]
    for name in dir(gg):
        k = getattr(gg, name)
        if hasattr(k, "configs") and name.startswith("_grouped"):
            k.configs = [k.configs[0]]
    import triton_moe.kernels as K

    K.fused_route = ns["fused_route"]
    return moe_mod, K, gg


def np32(t):
    return t.detach().cpu().numpy().copy()


def gen_route(K, torch):
    cases = {}
    rng = np.random.default_rng(1234)
    specs = [
        ("r0", 64, 4, 16, "up"),
        ("r1", 300, 8, 64, "up"),
        ("r2", 1000, 16, 128, "up"),
        ("r3", 513, 5, 32, "down"),
        ("r4", 513, 5, 32, "nearest"),
        ("r5", 40, 6, 64, "up"),  # some experts get no tokens
        ("r6", 2048, 64, 16, "up"),
    ]
    for name, A, E, bs, rounding in specs:
        sel = rng.integers(0, E if name != "r5" else 3, size=A).astype(np.int64)
        out = K.fused_route(torch.from_numpy(sel), E, block_size=bs, rounding=rounding)
        d = dict(sel=sel, E=np.int64(E), bs=np.int64(bs), rounding=np.array(rounding))
        for key, v in zip(("bin_ids", "indices", "tokens_per_expert", "bins", "padded_bins"), out):
            d[key] = np32(v).astype(np.int32)
        cases[name] = d
    np.savez_compressed(OUT / "route.npz", **{f"{c}__{k}": v for c, d in cases.items() for k, v in d.items()})


def gen_permute(K, torch):
    g = torch.Generator().manual_seed(7)
    T, k, E, H, bs = 24, 2, 4, 40, 16
    sel = torch.randint(0, E, (T * k,), generator=g)
    bin_ids, indices, tpe, bins, padded_bins = K.fused_route(sel, E, block_size=bs)
    x = torch.randn(T, H, generator=g)
    w = torch.rand(T * k, generator=g)
    xg = K.padded_gather(x, indices, bin_ids, bins, padded_bins, k)
    from triton_moe.kernels.gather import _weighted_padded_gather

    gxw = _weighted_padded_gather(x, indices, bin_ids, w, bins, padded_bins, k)
    y = torch.randn(xg.shape[0], H, generator=g)
    sc = K.padded_scatter(y, indices, bin_ids, w, bins, padded_bins, k)
    gm = K.precompute_gather_map(indices, bin_ids, bins, padded_bins, k)
    np.savez_compressed(
        OUT / "permute.npz",
        sel=sel.numpy(), top_k=np.int64(k), E=np.int64(E), bs=np.int64(bs),
        bin_ids=np32(bin_ids), indices=np32(indices), bins=np32(bins), padded_bins=np32(padded_bins),
        x=np32(x), w=np32(w), y=np32(y), gathered=np32(xg), weighted_gathered=np32(gxw),
        scattered=np32(sc), gather_map=np32(gm),
    )


def gen_gemm(K, torch):
    cases = {}
    g = torch.Generator().manual_seed(11)
    specs = [("uniform", 32, [64, 64, 64], [32, 0, 64]), ("variable", 48, [128, 32, 64], [64, 32, 48])]
    for name, H, widths, counts in specs:
        E = len(widths)
        tok_off = torch.tensor([0] + list(np.cumsum(counts)), dtype=torch.int32)
        w_off = torch.tensor([0] + list(np.cumsum(widths)), dtype=torch.int32)
        widths_t = torch.tensor(widths, dtype=torch.int32)
        tpe = torch.tensor(counts, dtype=torch.int32)
        P, TW, maxw = int(tok_off[-1]), int(w_off[-1]), max(widths)
        x = torch.randn(P, H, generator=g)
        w1 = torch.randn(H, TW, generator=g) * 0.1
        w2 = torch.randn(TW, H, generator=g) * 0.1
        out, pre = K.grouped_gemm_up(x, w1, tok_off, w_off, widths_t, tpe, maxw,
                                     activation="relu_squared", save_pre_act=True)
        out_none = K.grouped_gemm_up(x, w1, tok_off, w_off, widths_t, tpe, maxw, activation="none")
        y = K.grouped_gemm_down(out, w2, tok_off, w_off, widths_t, tpe, H)
        gy = torch.randn(P, H, generator=g)
        gi, gw2 = K.grouped_gemm_down_backward(gy, out, w2, tok_off, w_off, widths_t, tpe, H, maxw)
        gx, gw1 = K.grouped_gemm_up_backward(gi, x, w1, pre, tok_off, w_off, widths_t, tpe, H,
                                             "relu_squared")
        # fused-gather variant: x_flat + gather_map (gather_map rows are a permutation here)
        T = P // 2
        x_flat = torch.randn(T, H, generator=g)
        gmap = torch.randint(0, T, (P,), generator=g, dtype=torch.int32)
        out_gm = K.grouped_gemm_up(x_flat, w1, tok_off, w_off, widths_t, tpe, maxw,
                                   activation="relu_squared", gather_map=gmap)
        gx_gm, gw1_gm = K.grouped_gemm_up_backward(gi, x_flat, w1, pre, tok_off, w_off, widths_t,
                                                   tpe, H, "relu_squared", gather_map=gmap)
        d = dict(H=np.int64(H), widths=np.array(widths), counts=np.array(counts), tok_off=np32(tok_off),
                 w_off=np32(w_off), x=np32(x), w1=np32(w1), w2=np32(w2), out=np32(out), pre=np32(pre),
                 out_none=np32(out_none), y=np32(y), gy=np32(gy), gi=np32(gi), gw2=np32(gw2),
                 gx=np32(gx), gw1=np32(gw1), x_flat=np32(x_flat), gmap=np32(gmap),
                 out_gm=np32(out_gm), gx_gm=np32(gx_gm), gw1_gm=np32(gw1_gm))
        cases[name] = d
    np.savez_compressed(OUT / "gemm.npz", **{f"{c}__{k}": v for c, d in cases.items() for k, v in d.items()})


def gen_swiglu(K, torch):
    """The reference's swiglu up projection (forward only: its backward is a
    placeholder).  w1 holds each expert's gate block then its up block."""
    cases = {}
    g = torch.Generator().manual_seed(13)
    for name, H, widths, counts in [("variable", 48, [64, 32, 48], [64, 32, 48]),
                                    ("uniform", 32, [32, 32], [48, 0])]:
        tok_off = torch.tensor([0] + list(np.cumsum(counts)), dtype=torch.int32)
        w_off = torch.tensor([0] + list(np.cumsum([2 * w for w in widths])), dtype=torch.int32)
        widths_t = torch.tensor(widths, dtype=torch.int32)
        tpe = torch.tensor(counts, dtype=torch.int32)
        P, TW, maxw = int(tok_off[-1]), int(w_off[-1]), max(widths)
        x = torch.randn(P, H, generator=g)
        w1 = torch.randn(H, TW, generator=g) * 0.1
        out, pre = K.grouped_gemm_up(x, w1, tok_off, w_off, widths_t, tpe, maxw,
                                     activation="swiglu", save_pre_act=True)
        cases[name] = dict(H=np.int64(H), widths=np.array(widths), counts=np.array(counts),
                           tok_off=np32(tok_off), w_off=np32(w_off), x=np32(x), w1=np32(w1),
                           out=np32(out), pre=np32(pre))
    np.savez_compressed(OUT / "swiglu.npz",
                        **{f"{c}__{k}": v for c, d in cases.items() for k, v in d.items()})


def gen_layer(moe_mod, torch):
    """The small CPU config (n_embd 64, 4 experts x 128, top-2, 2 x 16 tokens), a
    variable-width variant, and variants without top-k renormalisation, with
    top-1 and with block size 128: full layer fwd + bwd."""
    from triton_moe import TritonMoEConfig, TritonMoEMLP

    cases = {}
    specs = [
        ("c1", dict(n_embd=64, expert_sizes=[(4, 128)], num_active_experts=2), 2, 16, 0),
        ("c1v", dict(n_embd=64, expert_sizes=[(2, 128), (2, 64)], num_active_experts=2), 2, 24, 1),
        ("c1n", dict(n_embd=64, expert_sizes=[(4, 128)], num_active_experts=2,
                     norm_topk_prob=False), 2, 16, 2),
        ("c1k1", dict(n_embd=64, expert_sizes=[(2, 128), (2, 64)], num_active_experts=1), 2, 16, 3),
        ("c1b", dict(n_embd=64, expert_sizes=[(4, 128)], num_active_experts=2, block_size=128),
         2, 16, 4),
    ]
    for name, cfg, B, S, seed in specs:
        torch.manual_seed(seed)
        m = TritonMoEMLP(TritonMoEConfig(**cfg)).float()
        with torch.no_grad():
            m.router.weight.normal_(0, 0.02)
            m.w1.normal_(0, 0.02)
            m.w2.normal_(0, 0.02)
        x = torch.randn(B, S, cfg["n_embd"], requires_grad=True)
        inter = m.forward_with_intermediates(x)
        out, aux, f_i = m(x)
        out.sum().backward()
        cases[name] = dict(
            n_embd=np.int64(cfg["n_embd"]),
            expert_sizes=np.array(cfg["expert_sizes"]),
            top_k=np.int64(cfg["num_active_experts"]),
            block_size=np.int64(m.block_size),
            norm_topk_prob=np.int64(bool(m.norm_topk_prob)),
            router_w=np32(m.router.weight), w1=np32(m.w1), w2=np32(m.w2), x=np32(x),
            selected=np32(inter["selected_experts_flat"]), weights=np32(inter["top_k_weights_flat"]),
            out=np32(out), dx=np32(x.grad), dw1=np32(m.w1.grad), dw2=np32(m.w2.grad),
            f_i=np32(f_i), z_loss=np32(aux["router_z_loss"]), lb_loss=np32(aux["load_balance_loss"]),
            compute_loss=np32(aux["compute_loss"]),
        )
    np.savez_compressed(OUT / "layer.npz", **{f"{c}__{k}": v for c, d in cases.items() for k, v in d.items()})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout")
    ap.add_argument("--only", nargs="*", default=None,
                    help="generate only these files (route permute gemm swiglu layer)")
    a = ap.parse_args()
    moe_mod, K, gg = load_reference(a.ref)
    import torch

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gens = {"route": lambda: gen_route(K, torch), "permute": lambda: gen_permute(K, torch),
            "gemm": lambda: gen_gemm(K, torch), "swiglu": lambda: gen_swiglu(K, torch),
            "layer": lambda: gen_layer(moe_mod, torch)}
    for name, fn in gens.items():
        if a.only is None or name in a.only:
            fn()
    for p in sorted(OUT.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
