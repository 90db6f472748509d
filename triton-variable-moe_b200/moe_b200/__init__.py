"""B200-native (sm_100a) MoE MLP hot path, a drop-in for triton_moe.

    from moe_b200 import TritonMoEConfig, TritonMoEMLP
    from moe_b200.kernels import grouped_gemm_up_autograd, ...

`install_as_triton_moe()` registers this package under the reference's import
names (`triton_moe`, `triton_moe.kernels`, `triton_moe.moe`) so existing code
that imports triton_moe runs on these kernels unchanged.
"""

import sys

from . import kernels
from .moe import TritonMoEConfig, TritonMoEMLP

__all__ = ["TritonMoEConfig", "TritonMoEMLP", "ExpertParallelMoEMLP", "install_as_triton_moe"]


def __getattr__(name):
    if name == "ExpertParallelMoEMLP":  # needs torch.distributed; imported on demand
        from .ep import ExpertParallelMoEMLP

        return ExpertParallelMoEMLP
    raise AttributeError(name)


def install_as_triton_moe() -> None:
    """Alias this package as `triton_moe` in sys.modules."""
    from . import moe as _moe

    sys.modules["triton_moe"] = sys.modules[__name__]
    sys.modules["triton_moe.kernels"] = kernels
    sys.modules["triton_moe.moe"] = _moe
