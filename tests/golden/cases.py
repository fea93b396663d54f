"""Golden-vector cases: small seeded problems on which the reference's own CPU path was
run (tests/golden/make_golden.py) to pin the oracle.  Test infrastructure."""
from __future__ import annotations

import hashlib

import torch

# name, M, H, N, dtype, seed, has_residual, eps
CASES = [
    # configs[0] of the benchmark spec: 4 tokens, H=256, 4 q + 2 kv heads of 64 -> N=512, fp32.
    dict(name="cpu_ref_fp32", M=4, H=256, N=512, dtype=torch.float32, seed=1, res=True, eps=1e-5),
    dict(name="bf16_m16_gqa", M=16, H=256, N=512, dtype=torch.bfloat16, seed=2, res=True, eps=1e-5),
    dict(name="fp16_m8_mha", M=8, H=256, N=768, dtype=torch.float16, seed=3, res=True, eps=1e-6),
    dict(name="bf16_m5_nores", M=5, H=512, N=640, dtype=torch.bfloat16, seed=4, res=False, eps=1e-5),
    dict(name="bf16_m3_ragged", M=3, H=264, N=200, dtype=torch.bfloat16, seed=5, res=True, eps=1e-6),
    dict(name="fp16_m33_gqa", M=33, H=512, N=768, dtype=torch.float16, seed=6, res=True, eps=1e-5),
]


def as_bits(t: torch.Tensor):
    """Raw bit pattern of a tensor as a numpy array (uint16 for 16-bit floats)."""
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.view(torch.int16).numpy().view("uint16")
    return t.numpy()


def inputs_digest(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        if t is not None:
            h.update(as_bits(t).tobytes())
    return h.hexdigest()
