"""B200-native (sm_100a) NVFP4 SwiGLU mixture-of-experts layer.

Drop-in for the ``SparseMoE`` hot path of mESmaC/MCL4-COE
(src/mcl4_coe/backbone.py:190-1047) and its NVFP4 operator seam
(src/mcl4_coe/nvfp4.py).  The compute runs in ``libmcl4moe.so`` (hand-written
CUDA for sm_100a behind the C ABI of ``include/mcl4moe.h``); this package is
the thin PyTorch host side.  The directory name contains a dash, so import it
through ``__graft_entry__.load_package()`` (registered as ``mcl4coe_b200``).
"""

from . import _lib, routing_variants
from .expert_parallel import CudaEPOps, ExpertParallelMoE
from .moe import MoEConfig, SparseMoE, SwiGLUExpert
from .nvfp4 import (
    SPARSITY_MODES,
    GroupedNVFP4Cache,
    compute_2to4_mask,
    export_reference_cache,
    get_gemm_counts,
    get_or_build_grouped_cache,
    NVFP4Linear,
    convert_linear_to_nvfp4,
    nvfp4_grouped_linear,
    nvfp4_mm,
    quantize_activations,
    quantize_nvfp4,
    reset_gemm_counts,
)

__all__ = [
    "CudaEPOps",
    "ExpertParallelMoE",
    "MoEConfig",
    "SparseMoE",
    "SwiGLUExpert",
    "GroupedNVFP4Cache",
    "export_reference_cache",
    "get_gemm_counts",
    "get_or_build_grouped_cache",
    "nvfp4_grouped_linear",
    "quantize_nvfp4",
    "reset_gemm_counts",
    "compute_2to4_mask",
    "SPARSITY_MODES",
    "NVFP4Linear",
    "convert_linear_to_nvfp4",
    "nvfp4_mm",
    "quantize_activations",
]


def library():
    """Load (once) and return the ctypes handle of ``libmcl4moe.so``."""
    return _lib.load()
