"""B200-native fused residual add + RMSNorm + packed QKV projection.

Import-compatible with the reference package ``triton_fused_rmsnorm_qkv``
(``src/triton_fused_rmsnorm_qkv/__init__.py:1-17``): the same six names, plus
``fused_add_rmsnorm_matmul`` (returns the updated residual as well) and
``qkv_rope_split`` (head-major Q/K/V with the rotary embedding, one launch).  The GPU entry
points run sm_100a CUDA kernels from ``libfqkv.so``; they raise if that library is
missing instead of falling back to anything else.
"""
from .baseline import rmsnorm_residual_qkv
from .kernel import (
    device_status,
    fused_add_rmsnorm_matmul,
    fused_rmsnorm_residual_matmul,
    fused_rmsnorm_residual_matmul_fixed,
    fused_rmsnorm_residual_qkv,
    fused_rmsnorm_residual_qkv_fixed,
    get_autotune_best_config,
    qkv_rope_split,
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
]
