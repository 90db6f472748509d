"""sm_100a kernel wrappers with the export list of triton_moe.kernels
(triton_moe/kernels/__init__.py:18-40)."""

from ._ops import check_device_status
from .fused_cumsum import fused_route
from .gather import padded_gather, padded_gather_autograd
from .grouped_gemm import (
    GroupedGemmDown,
    GroupedGemmUp,
    grouped_gemm_down,
    grouped_gemm_down_autograd,
    grouped_gemm_down_backward,
    grouped_gemm_up,
    grouped_gemm_up_autograd,
    grouped_gemm_up_backward,
    precompute_gather_map,
)
from .scatter import padded_scatter, padded_scatter_autograd

__all__ = [
    # Gather/Scatter
    "padded_gather",
    "padded_gather_autograd",
    "padded_scatter",
    "padded_scatter_autograd",
    # Forward kernels
    "grouped_gemm_up",
    "grouped_gemm_down",
    # Backward kernels
    "grouped_gemm_up_backward",
    "grouped_gemm_down_backward",
    # Autograd wrappers
    "grouped_gemm_up_autograd",
    "grouped_gemm_down_autograd",
    # Gather map for fused gather
    "precompute_gather_map",
    # Autograd Function classes
    "GroupedGemmUp",
    "GroupedGemmDown",
    # Routing
    "fused_route",
    # Device status word (bounded waits, bad expert ids, capacity)
    "check_device_status",
]
