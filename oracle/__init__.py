"""Test infrastructure: the CPU oracle for the fused residual add + RMSNorm + QKV path.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
use this package, and only as the checker / the timed CPU reference.  The product
(``triton_fused_rmsnorm_qkv``) never imports it.
"""
from .rmsnorm_qkv import (  # noqa: F401
    faithful_rounding_metrics,
    forward,
    make_case,
    parity_metrics,
    project,
    residual_add,
    rms_normalize,
    split_qkv,
    ulp,
    within_bars,
)
from .rope import make_rope_case, rope_split  # noqa: F401,E402
from .fp8w import forward_fp8w  # noqa: F401,E402
