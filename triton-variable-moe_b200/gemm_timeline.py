"""Per-CTA timeline of the grouped-GEMM launches of one training step.

Needs the timeline build of the library (`python build.py --trace`, which
writes moe_b200/libmoe_b200_trace.so with -DMOE_TRACE).  Runs bench.py's
layer for a config, one launch at a time (synchronised, L2 flushed before
each step), reads every CTA's %globaltimer stamps after each GEMM launch and
prints, per launch, the spread of CTA start/end times and, for each of a
CTA's first tiles, when its producer began, its MMA issuer started and
finished the tile, and its epilogue finished, plus the first CTAs' per
k-block load issue / landing times.

    python triton-variable-moe_b200/gemm_timeline.py [c3|c4]
"""
import ctypes
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
os.environ["MOE_B200_LIB"] = os.path.join(HERE, "moe_b200", "libmoe_b200_trace.so")
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(HERE))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import bench  # noqa: E402
from moe_b200 import _lib  # noqa: E402

NAMES = ["moe_grouped_gemm_up_down", "moe_grouped_gemm_down_backward",
         "moe_grouped_gemm_up_backward"]


def main():
    cfgname = sys.argv[1] if len(sys.argv) > 1 else "c3"
    cfg = bench.CONFIGS[cfgname]
    dev = torch.device("cuda", 0)
    layer = bench.build_layer(cfg, dev)
    x_h, g_h = bench.make_tokens(cfg, 0)
    x = x_h.to(dev).requires_grad_(True)
    gout = g_h.to(dev)
    lib = _lib.lib
    rd = lib.moe_trace_read
    rd.argtypes = [ctypes.c_void_p]
    rd.restype = ctypes.c_int
    buf = np.zeros(2 * 160 * 64, dtype=np.uint64)
    traces = {}
    for n in NAMES:
        f = getattr(lib, n)

        def wrap(*a, _f=f, _n=n):
            torch.cuda.synchronize()
            rd(buf.ctypes.data)
            rc = _f(*a)
            torch.cuda.synchronize()
            rd(buf.ctypes.data)
            traces[_n] = buf.copy().reshape(2, 160, 64).astype(np.int64)
            return rc

        setattr(lib, n, wrap)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    for _ in range(4):
        flush.zero_()
        layer.zero_grad(set_to_none=True)
        x.grad = None
        out, _, _ = layer(x)
        out.backward(gout)
    torch.cuda.synchronize()
    for n in NAMES:
        tr, kb = traces[n]
        ctas = np.nonzero(tr[:, 0])[0]
        t0 = tr[ctas, 0].min()
        us = lambda v: (v - t0) / 1000.0  # noqa: E731
        end = us(tr[ctas, 2])
        print(f"== {n}: {len(ctas)} CTAs; after griddep wait {np.median(us(tr[ctas, 1])):.2f} us; "
              f"end median {np.median(end):.2f} max {end.max():.2f} us")
        ntiles = np.array([sum(1 for i in range(8) if tr[c, 3 + 7 * i]) for c in ctas])
        first_load = us(tr[ctas, 3])
        print("  CTA end percentiles (10/25/50/75/90/100):",
              " ".join(f"{np.percentile(end, q):.2f}" for q in (10, 25, 50, 75, 90, 100)),
              f"| first tile's producer begin min {first_load.min():.2f} "
              f"median {np.median(first_load):.2f}",
              "| tiles per CTA:", dict(zip(*np.unique(ntiles, return_counts=True))))
        marks = {s: tr[ctas, s] for s in (59, 60, 61, 62)}
        print("  producer after the fence point / launch_dependents / table read / first tile decoded (median):",
              " ".join(f"{np.median(us(v[v != 0])):.2f}" if (v != 0).any() else "-"
                       for v in marks.values()))
        for i in range(4):
            cols = [3 + 7 * i + e for e in range(7)]
            sub = tr[ctas][:, cols]
            ok = sub[:, 0] != 0
            if not ok.any():
                break
            r = us(sub[ok])
            med = lambda a: f"{np.median(a):6.2f}"  # noqa: E731
            print(f"  tile {i} ({ok.sum()} CTAs): producer begin {med(r[:, 0])}  mma start "
                  f"{med(r[:, 3])} end {med(r[:, 4])}  epilogue from {med(r[:, 5])} to "
                  f"{med(r[:, 6])}")
        for c in ctas[:2]:
            iss = [us(v) for v in kb[c, :32] if v]
            land = [us(v) for v in kb[c, 32:] if v]
            print(f"  cta {c} k-block issue:", " ".join(f"{v:.2f}" for v in iss[:12]))
            print(f"  cta {c} k-block land :", " ".join(f"{v:.2f}" for v in land[:12]))


if __name__ == "__main__":
    main()
