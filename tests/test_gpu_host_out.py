"""Results written by the kernel straight into page-locked host memory (``out=`` /
``residual_out=`` pinned host tensors) on the schedules that store with plain stores: the
host copy read after a stream synchronisation must equal the device-output call bit for
bit, and match the CPU oracle; calls in a row reuse the same host buffers.  Pageable host
memory and the schedules that store through TMA are rejected before any launch."""
from __future__ import annotations

import pytest
import torch

from oracle import forward, make_case, parity_metrics, within_bars
from triton_fused_rmsnorm_qkv import fused_add_rmsnorm_matmul

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,H,N,dtype,res,sched", [
    (16, 4096, 6144, torch.bfloat16, True, None),    # decode (cluster kernel), Llama-3-8B
    (1, 3584, 4608, torch.bfloat16, True, None),     # Qwen2-7B M=1: grid schedule
    (7, 1024, 1280, torch.float16, False, "decode"),
    (5, 100, 72, torch.bfloat16, True, None),        # unaligned H: simt
])
def test_host_outputs_equal_device_outputs(M, H, N, dtype, res, sched):
    out_h = torch.empty(1, M, N, dtype=dtype).pin_memory()
    hid_h = torch.empty(1, M, H, dtype=dtype).pin_memory()
    for call in range(3):
        x, r, g, w = make_case(M, H, N, dtype, seed=40 + call, has_residual=res)
        xd, rd, gd, wd = (t.cuda() if t is not None else None for t in (x, r, g, w))
        o_dev, h_dev = fused_add_rmsnorm_matmul(xd[None], rd[None] if res else None, gd, wd, 1e-5, schedule=sched)
        fused_add_rmsnorm_matmul(xd[None], rd[None] if res else None, gd, wd, 1e-5, schedule=sched, out=out_h,
                                 residual_out=hid_h)
        torch.cuda.synchronize()
        assert torch.equal(out_h, o_dev.cpu()), call
        assert torch.equal(hid_h, h_dev.cpu()), call
        ref_out, ref_hidden = forward(x, r, g, w, 1e-5)
        assert within_bars(parity_metrics(out_h[0].clone(), ref_out)), call
        assert torch.equal(hid_h[0], ref_hidden), call


def test_host_outputs_rejected_where_they_cannot_be_written():
    M, H, N = 16, 1024, 1536
    x, r, g, w = (t.cuda() for t in make_case(M, H, N, torch.bfloat16, seed=3))
    with pytest.raises(ValueError, match="page-locked"):
        fused_add_rmsnorm_matmul(x[None], r[None], g, w, 1e-5, out=torch.empty(1, M, N, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="decode, grid or simt"):
        fused_add_rmsnorm_matmul(x[None], r[None], g, w, 1e-5, schedule="prefill",
                                 out=torch.empty(1, M, N, dtype=torch.bfloat16).pin_memory())
