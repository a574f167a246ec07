"""B200-native (sm_100a) W4A8 Mixture-of-Experts grouped GEMM.

Drop-in for the ``w4a8_group_gemm_moe`` operator of CaiJichang212/flagos-kernel-gen
(docs/Task1.md:8-17), plus the routed MoE layer around it and an
expert-parallel mode.  All compute runs in the in-tree CUDA library
``lib/libw4a8moe.so`` through its C ABI (include/w4a8moe.h); importing this
package does not touch the GPU.

The directory name is not a Python identifier, so import it with
``importlib.import_module("flagos-kernel-gen_b200")``.
"""
from .ops import (  # noqa: F401
    AlignResult,
    act_quant,
    align_capacity,
    combine_finish,
    device_status,
    gather_rows,
    moe_align,
    moe_combine,
    prepack_weights,
    quant_scatter,
    router_topk,
    silu_mul_requant,
    w4a8_group_gemm_moe,
    w4a8_group_gemm_moe_combine,
    w4a8_group_gemm_moe_ex,
)
from .moe import HostPipeline, MoELayer, W4A8Weights, w4a8_moe  # noqa: F401
from ._lib import KERNEL_AUTO, KERNEL_GEMV, KERNEL_SIMT, KERNEL_TC  # noqa: F401
from . import ops, workloads  # noqa: F401

__all__ = [
    "w4a8_group_gemm_moe", "w4a8_group_gemm_moe_ex", "w4a8_group_gemm_moe_combine", "combine_finish", "act_quant", "moe_align", "quant_scatter",
    "router_topk", "prepack_weights", "silu_mul_requant", "moe_combine", "gather_rows", "device_status", "MoELayer", "HostPipeline", "W4A8Weights",
    "w4a8_moe",
    "KERNEL_AUTO", "KERNEL_TC", "KERNEL_SIMT", "KERNEL_GEMV", "ops", "workloads",
]
