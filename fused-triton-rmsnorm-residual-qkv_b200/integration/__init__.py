"""Model integrations of the fused RMSNorm + QKV op (the reference's ``integration``
package, ``integration/__init__.py:1-15``)."""
from .decode import GraphedGreedyDecoder
from .llama3_patch import (
    LLAMA3_8B_CONFIG,
    apply_fused_patch,
    build_llama3_8b,
    fused_patch,
    remove_fused_patch,
)

__all__ = [
    "GraphedGreedyDecoder",
    "LLAMA3_8B_CONFIG",
    "build_llama3_8b",
    "apply_fused_patch",
    "remove_fused_patch",
    "fused_patch",
]
