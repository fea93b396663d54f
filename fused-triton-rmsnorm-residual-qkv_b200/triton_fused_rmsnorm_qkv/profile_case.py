"""A small, fixed workload of the fused op for a profiler capture.

    python -m triton_fused_rmsnorm_qkv.profile_case --H 3584 --N 4608 --M 1 --schedule grid
    ncu --set full --clock-control none -k regex:decode_kernel -s 4 -c 1 -o prof \\
        python -m triton_fused_rmsnorm_qkv.profile_case --H 3584 --N 4608 --M 1 --schedule grid

Seeded x / residual ~ N(0, 1), gains 1 + 0.1 N(0, 1) and weights N(0, 0.02) on the first CUDA
device; ``--calls`` calls of ``fused_add_rmsnorm_matmul`` (or, with ``--fp8w``,
``fused_add_rmsnorm_matmul_fp8w`` on weights quantised by ``quantize_weight_e4m3``) rotate
over ``--sets`` weight sets, so that with weights larger than a quarter of L2 each captured
launch reads its weight from HBM.  Prints one line with a checksum of the last output.
"""
from __future__ import annotations

import argparse

import torch

from . import fused_add_rmsnorm_matmul, fused_add_rmsnorm_matmul_fp8w, quantize_weight_e4m3


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--H", type=int, default=4096)
    ap.add_argument("--N", type=int, default=6144)
    ap.add_argument("--M", type=int, default=16)
    ap.add_argument("--schedule", default=None, help="auto (default), decode, grid, split, prefill or simt")
    ap.add_argument("--dtype", choices=("bf16", "fp16"), default="bf16")
    ap.add_argument("--fp8w", action="store_true", help="e4m3 weights with an fp32 scale per row")
    ap.add_argument("--sets", type=int, default=4)
    ap.add_argument("--calls", type=int, default=8)
    a = ap.parse_args(argv)
    dt = torch.bfloat16 if a.dtype == "bf16" else torch.float16
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    sets = []
    for _ in range(a.sets):
        gain = (1 + 0.1 * torch.randn(a.H, generator=g, device=dev)).to(dt)
        w = (0.02 * torch.randn(a.N, a.H, generator=g, device=dev)).to(dt)
        sets.append((gain, quantize_weight_e4m3(w) if a.fp8w else w))
    x = torch.randn(1, a.M, a.H, generator=g, device=dev).to(dt)
    r = torch.randn(1, a.M, a.H, generator=g, device=dev).to(dt)
    out = None
    for i in range(a.calls):
        gain, w = sets[i % a.sets]
        if a.fp8w:
            out, _ = fused_add_rmsnorm_matmul_fp8w(x, r, gain, w[0], w[1], 1e-5, static_weights=True)
        else:
            out, _ = fused_add_rmsnorm_matmul(x, r, gain, w, 1e-5, schedule=a.schedule, static_weights=True)
    torch.cuda.synchronize()
    print(f"ok M={a.M} H={a.H} N={a.N} calls={a.calls} checksum={float(out.float().abs().sum()):.6e}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
