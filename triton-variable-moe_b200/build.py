"""Build libmoe_b200.so (all CUDA kernels + the C ABI) in-tree for sm_100a.

Usage: python triton-variable-moe_b200/build.py [--force] [-j N]

The library is written next to the Python package
(moe_b200/libmoe_b200.so) so it travels with the source tree.  Objects are
rebuilt only when a source or header is newer than the object.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OBJ_DIR = HERE / "_build"
OUT = HERE / "moe_b200" / "libmoe_b200.so"

SOURCES = ["route.cu", "router.cu", "permute.cu", "grouped_gemm.cu", "capi.cu", "ep.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    *ARCH,
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, obj: Path, extra: list[str]) -> None:
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    subprocess.run(cmd, check=True)


def build(force: bool = False, jobs: int = 4, verbose_ptxas: bool = False,
          trace: bool = False) -> Path:
    """Compile the library.  trace=True builds the GEMM timeline variant
    (-DMOE_TRACE, exports moe_trace_read) as libmoe_b200_trace.so instead."""
    obj_dir = OBJ_DIR.with_name("_build_trace") if trace else OBJ_DIR
    out = OUT.with_name("libmoe_b200_trace.so") if trace else OUT
    obj_dir.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    if trace:
        extra.append("-DMOE_TRACE")
    todo = []
    objs = []
    for s in SOURCES:
        src = CSRC / s
        obj = obj_dir / (s + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            todo.append((src, obj))
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        list(ex.map(lambda so: _compile(so[0], so[1], extra), todo))
    if todo or force or not out.exists():
        # exported symbols: only the extern "C" ABI (default visibility below)
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(out), *map(str, objs), "-Xcompiler", "-fPIC",
               "-ldl"]
        subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=4)
    ap.add_argument("--ptxas-v", action="store_true")
    ap.add_argument("--trace", action="store_true", help="GEMM timeline build (-DMOE_TRACE)")
    a = ap.parse_args()
    print(build(a.force, a.j, a.ptxas_v, a.trace))
    sys.exit(0)
