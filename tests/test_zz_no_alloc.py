"""fqkv_launch_noalloc: the op for callers that cannot allocate device memory when they
run it -- an inference engine's plugin whose enqueue step must not allocate (the engine
owns all device memory, and cudaMalloc can synchronise the device), or a runtime with a
fixed memory budget that allocates nothing after start-up.  It runs the split schedule on
a fixed device array owned by the library instead of a caller workspace.

Each call's output is checked against the regular entry point's on the same inputs and
against the CPU oracle, with the tolerance of the other parity tests, on calls in a row:
the later calls reuse the array the earlier ones left behind, one of them with the same
shape as the first.  This file is collected last so that a failure here comes after every
other test has run.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import forward, make_case, parity_metrics, within_bars
from triton_fused_rmsnorm_qkv import _lib, fused_add_rmsnorm_matmul

pytestmark = pytest.mark.gpu


def _noalloc(x, r, g, w, eps):
    lib = _lib.load()
    fn = lib.fqkv_launch_noalloc
    i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    fn.argtypes = [vp, vp, vp, i32, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, i64, ctypes.c_float, i32, i32, vp]
    fn.restype = i32
    M, H = x.shape
    N = w.shape[0]
    out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    hidden = torch.empty_like(x)
    dt = _lib.BF16 if x.dtype == torch.bfloat16 else _lib.F16
    gdt = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}[g.dtype]
    rc = fn(x.data_ptr(), r.data_ptr() if r is not None else None, g.data_ptr(), gdt, w.data_ptr(), out.data_ptr(),
            hidden.data_ptr(), M, H, N, x.stride(0), r.stride(0) if r is not None else 0, w.stride(0), out.stride(0),
            hidden.stride(0), eps, dt, _lib.FLAG_PDL, torch.cuda.current_stream().cuda_stream)
    return rc, out, hidden


def test_noalloc_matches_regular_entry_point_on_calls_in_a_row():
    cases = [(16, 4096, 6144, torch.bfloat16, True, 1e-5, 50), (7, 1024, 1280, torch.float16, False, 1e-6, 51),
             (16, 4096, 6144, torch.bfloat16, True, 1e-5, 52)]  # the first shape again, new inputs
    for call, (M, H, N, dtype, res, eps, seed) in enumerate(cases):
        xc, rc_, gc, wc = make_case(M, H, N, dtype, seed=seed, has_residual=res)
        x, r, g, w = (t.cuda() if t is not None else None for t in (xc, rc_, gc, wc))
        rc, out, hidden = _noalloc(x, r, g, w, eps)
        assert rc == 0, _lib.last_error()
        ref_out, ref_hidden = fused_add_rmsnorm_matmul(x[None], r[None] if r is not None else None, g, w, eps,
                                                      schedule="split")
        torch.cuda.synchronize()
        m = parity_metrics(out.cpu(), ref_out[0].cpu())
        assert within_bars(m), (call, "vs fqkv_launch", m)
        assert torch.equal(hidden.cpu(), ref_hidden[0].cpu()), call
        oracle_out, oracle_hidden = forward(xc, rc_, gc, wc, eps)
        m = parity_metrics(out.cpu(), oracle_out)
        assert within_bars(m), (call, "vs oracle", m)
        assert torch.equal(hidden.cpu(), oracle_hidden), call


def test_noalloc_rejects_sizes_beyond_its_array():
    x, r, g, w = (t.cuda() for t in make_case(17, 256, 512, torch.bfloat16, seed=3))
    rc, _, _ = _noalloc(x, r, g, w, 1e-5)
    assert rc == _lib.ERR_SHAPE
    assert "fqkv_launch_noalloc takes M <= 16" in _lib.last_error()
