"""ctypes binding of libmoe_b200.so, the C ABI declared in include/moe_b200.h.

The shared library holds every CUDA kernel of this package.  There is no
fallback: if the library cannot be loaded, importing this module raises, and
every op that needs it fails loudly.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_int, c_int64, c_void_p
from pathlib import Path

import torch

_HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("MOE_B200_LIB", _HERE / "libmoe_b200.so"))

MOE_OK = 0
STATUS_TEXT = {
    -1: "invalid argument",
    -2: "unsupported configuration",
    -3: "CUDA error",
    -4: "device-side wait timed out",
    -5: "padded row capacity exceeded",
    -6: "expert id out of range",
    -7: "NCCL unavailable or an NCCL call failed",
}

DTYPE_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
ACT_CODE = {"none": 0, "relu_squared": 1, "swiglu": 2}
ROUND_CODE = {"up": 0, "down": 1, "nearest": 2}
TILE_PAIR = 0x200  # tile_n flag: 256-row tiles on SM pairs (2-CTA clusters)


def tile_ctas(n: int) -> int:
    """tile_n field capping the persistent GEMM grid at n CTAs (MOE_TILE_CTAS)."""
    return int(n) << 16

_P = c_void_p
_I = c_int
_L = c_int64

# name -> argtypes (all functions return int unless listed in _RESTYPE)
_SIGS = {
    "moe_version": [],
    "moe_set_wait_timeout_ns": [ctypes.c_uint64],
    "moe_status_string": [_I],
    "moe_route_workspace_bytes": [_L, _I],
    "moe_route": [_P, _I, _L, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _L, _P, _P, _L, _P, _P],
    "moe_route_no_alloc": [_P, _I, _L, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _L, _P, _P, _P],
    "moe_router_topk": [_P, _L, _I, _I, _I, _P, _I, _P, _P],
    "moe_router_head_workspace_floats": [_L, _I],
    "moe_router_head": [_P, _I, _L, _I, _I, _I, _P, _P, _P, _I, _P, _P, _P, _P],
    "moe_router_head_losses": [_P, _I, _L, _I, _I, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P,
                               _P, _P, _P],
    "moe_aux_losses": [_P, _L, _I, _P, _P, _I, _P, _P, _I, _P, _P, _P],
    "moe_build_row_map": [_P, _P, _P, _P, _L, _L, _P, _L, _P, _P, _P],
    "moe_gather_map": [_P, _L, _I, _P, _P],
    "moe_padded_gather": [_P, _L, _L, _P, _I, _L, _P, _P, _P, _L, _I, _P],
    "moe_padded_scatter": [_P, _L, _L, _P, _L, _I, _P, _P, _L, _I, _P],
    "moe_relu_squared_grad": [_P, _P, _L, _L, _L, _P, _I, _P],
    "moe_grouped_gemm_up": [_P, _L, _L, _P, _L, _L, _P, _P, _P, _I, _I, _P, _P, _L, _I, _I, _P, _P],
    "moe_grouped_gemm_up_swiglu": [_P, _L, _L, _P, _L, _L, _P, _P, _P, _I, _P, _P, _P, _L, _I, _I,
                                   _P, _P],
    "moe_swiglu_grad": [_P, _P, _P, _L, _L, _P, _P, _I, _P, _L, _I, _P],
    "moe_up_down_dep_words": [_L, _I],
    "moe_grouped_gemm_up_down": [_P, _L, _L, _P, _P, _L, _L, _P, _P, _P, _I, _P, _P, _L, _P, _L, _P,
                                 _L, _I, _I, _I, _P, _P],
    "moe_grouped_gemm_down": [_P, _L, _L, _P, _L, _L, _P, _P, _P, _I, _P, _L, _I, _I, _P, _P],
    "moe_grouped_gemm_up_dx": [_P, _L, _L, _P, _L, _L, _P, _P, _P, _I, _P, _L, _I, _I, _P, _P],
    "moe_grouped_gemm_up_dw": [_P, _L, _L, _P, _L, _L, _L, _P, _P, _I, _P, _I, _I, _P, _P],
    "moe_grouped_gemm_down_dinter": [
        _P, _L, _L, _P, _L, _L, _P, _P, _P, _I, _P, _L, _P, _L, _I, _I, _P, _P,
    ],
    "moe_grouped_gemm_down_backward": [
        _P, _L, _L, _P, _L, _P, _L, _L, _P, _P, _P, _I, _P, _L, _P, _L, _P, _I, _I, _I, _P, _P,
    ],
    "moe_grouped_gemm_up_backward": [
        _P, _L, _L, _P, _L, _P, _L, _L, _P, _P, _P, _I, _P, _L, _P, _I, _I, _I, _P, _P,
    ],
    "moe_grouped_gemm_down_dw": [_P, _L, _L, _P, _L, _L, _L, _P, _P, _I, _P, _I, _I, _P, _P],
    "moe_ep_unique_id": [_P],
    "moe_ep_comm_init": [_P, _P, _I, _I],
    "moe_ep_comm_destroy": [_P],
    "moe_ep_gather_counts": [_P, _P, _P, _L, _P],
    "moe_ep_barrier": [_P, _P, _P],
    "moe_ep_buffer_create": [_L, _P, _P],
    "moe_ep_buffer_free": [_P],
    "moe_ep_buffer_open": [_P, _P],
    "moe_ep_buffer_close": [_P],
    "moe_ep_plan": [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P],
    "moe_ep_dispatch": [_P, _L, _L, _P, _I, _P, _P, _L, _P, _P, _P, _L, _I, _P],
    "moe_ep_combine": [_P, _L, _P, _P, _P, _P, _L, _I, _P, _L, _P, _L, _I, _P],
}
_RESTYPE = {
    "moe_version": c_char_p,
    "moe_set_wait_timeout_ns": ctypes.c_uint64,
    "moe_status_string": c_char_p,
    "moe_route_workspace_bytes": c_int64,
    "moe_router_head_workspace_floats": c_int64,
    "moe_up_down_dep_words": c_int64,
}

EXPORTED = tuple(_SIGS)


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"moe_b200: CUDA library {LIB_PATH} not found; build it with "
            "`python triton-variable-moe_b200/build.py` (or __graft_entry__.build())"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, args in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, c_int)
    return lib


lib = _load()


class MoEKernelError(RuntimeError):
    """A libmoe_b200 entry point returned a non-zero status."""


def check(rc: int, name: str) -> None:
    if rc != MOE_OK:
        raise MoEKernelError(f"{name} failed: {STATUS_TEXT.get(rc, rc)} (status {rc})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("moe_b200 kernels need CUDA tensors (no CPU fallback)")


def version() -> str:
    return lib.moe_version().decode()
