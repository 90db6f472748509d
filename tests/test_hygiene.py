"""Static checks of the product tree and of the bench's work accounting (CPU)."""

import ast
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "triton-variable-moe_b200"


def test_product_never_imports_the_oracle():
    """The oracle is test infrastructure: nothing in the package imports it, so
    the product path cannot fall back to it."""
    offenders = []
    for f in PKG.rglob("*.py"):
        tree = ast.parse(f.read_text(), filename=str(f))
        for node in ast.walk(tree):
            names = []
            if isinstance(node, ast.Import):
                names = [a.name for a in node.names]
            elif isinstance(node, ast.ImportFrom):
                names = [node.module or ""]
            if any(n == "oracle" or n.startswith("oracle.") for n in names):
                offenders.append(f"{f.relative_to(ROOT)}:{node.lineno}")
    assert not offenders, offenders


def test_bench_work_accounting():
    """GEMM FLOPs = 12 H sum_e n_e w_e over unpadded counts; permutation bytes =
    4 (T + A) H e + 2 A e (gather/scatter and their backward mirrors, weights)."""
    sys.path.insert(0, str(ROOT))
    import bench

    cfg = bench.CONFIGS["c3"]
    widths = bench.widths_of(cfg)
    assert widths == [512] * 4 + [256] * 8 + [128] * 4
    T = cfg["batch"] * cfg["seq"]
    A = T * cfg["top_k"]
    uniform = [A // len(widths)] * len(widths)
    flops = bench.gemm_flops(uniform, cfg)
    assert flops == 12 * 768 * sum(n * w for n, w in zip(uniform, widths))
    assert abs(flops / 1e9 - 43.5) < 0.1  # the c3 uniform-routing figure
    pb = bench.permute_bytes(cfg)
    assert pb == 4 * (T + A) * 768 * 2 + 2 * A * 2
    assert abs(pb / 1e6 - 151.06) < 0.01
