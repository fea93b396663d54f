"""B200-native fused residual add + RMSNorm + packed QKV projection.

Import-compatible with the reference package ``triton_fused_rmsnorm_qkv``
(``src/triton_fused_rmsnorm_qkv/__init__.py:1-17``): the same six names, plus
``fused_add_rmsnorm_matmul`` (returns the updated residual as well) and
``qkv_rope_split`` (head-major Q/K/V with the rotary embedding, one launch) and
``fused_add_rmsnorm_matmul_fp8w`` (e4m3 weights with a scale per row, decode sizes) and
``schedule_info`` (the schedule an automatic call of a shape runs).  The GPU entry
points run sm_100a CUDA kernels from ``libfqkv.so``; they raise if that library is
missing instead of falling back to anything else.
"""
from .baseline import rmsnorm_residual_qkv
from .kernel import (
    device_status,
    fused_add_rmsnorm_matmul,
    fused_add_rmsnorm_matmul_fp8w,
    fused_rmsnorm_residual_matmul,
    fused_rmsnorm_residual_matmul_fixed,
    fused_rmsnorm_residual_qkv,
    fused_rmsnorm_residual_qkv_fixed,
    get_autotune_best_config,
    qkv_rope_split,
    fused_add_rmsnorm_qkv_rope,
    quantize_weight_e4m3,
    schedule_info,
)

__all__ = [
    "rmsnorm_residual_qkv",
    "fused_rmsnorm_residual_matmul",
    "fused_rmsnorm_residual_matmul_fixed",
    "fused_rmsnorm_residual_qkv",
    "fused_rmsnorm_residual_qkv_fixed",
    "get_autotune_best_config",
    "fused_add_rmsnorm_matmul",
    "device_status",
    "qkv_rope_split",
    "fused_add_rmsnorm_qkv_rope",
    "fused_add_rmsnorm_matmul_fp8w",
    "quantize_weight_e4m3",
    "schedule_info",
]
