"""The Python layer's automatic choice of the grid schedule, on the CPU.

``kernel._grid_preferred`` takes ``grid`` when the rows are few (M <= 2), the library's own
choice is the cluster decode kernel, and the grid configuration streams at most 0.6x the
cluster configuration's weight k-blocks per CTA.  The library's schedule records are faked
here with the configurations it reports on a 148-SM B200, so only the rule is under test.
"""
from __future__ import annotations

import pytest

from triton_fused_rmsnorm_qkv import _lib
from triton_fused_rmsnorm_qkv import kernel as fk


def info(schedule, nt, split, grid):
    return {"schedule": schedule, "block_m": 16, "block_n": 128 * nt, "block_k": 64, "stages": 4, "split_k": split,
            "grid": grid, "threads": 320, "smem_bytes": 200000, "uses_prepass": 0}


# (H, N) -> (cluster record, grid record) as reported on a 148-SM B200.
RECORDS = {
    (3584, 4608): (info(_lib.SCHED_DECODE, 2, 6, 108), info(_lib.SCHED_GRID, 1, 4, 144)),    # 20 vs 14 k-blocks
    (4096, 6144): (info(_lib.SCHED_DECODE, 2, 5, 120), info(_lib.SCHED_GRID, 1, 3, 144)),    # 26 vs 22
    (8192, 10240): (info(_lib.SCHED_DECODE, 2, 3, 120), info(_lib.SCHED_GRID, 4, 7, 140)),   # 86 vs 76
    (4096, 28672): (info(_lib.SCHED_DECODE, 5, 3, 135), info(_lib.SCHED_GRID, 5, 3, 135)),   # equal
    (4096, 512): (info(_lib.SCHED_SPLIT, 1, 0, 148), info(_lib.SCHED_GRID, 1, 8, 32)),       # C picks split
    (2048, 8192): (info(_lib.SCHED_DECODE, 2, 2, 128), info(_lib.SCHED_GRID, 1, 4, 256)),   # 32 vs 8 (made up)
}


@pytest.fixture
def fake_library(monkeypatch):
    def query(M, H, N, dtype, schedule=_lib.SCHED_AUTO):
        cluster, grid = RECORDS[(H, N)]
        return grid if schedule == _lib.SCHED_GRID else cluster

    monkeypatch.setattr(fk._lib, "query_schedule", query)
    monkeypatch.setattr(fk, "_grid_choice", {})


@pytest.mark.parametrize("M,H,N,expect", [
    (1, 2048, 8192, True),     # a quarter of the bytes per CTA: 8 <= 0.6 x 32 k-blocks
    (2, 2048, 8192, True),
    (3, 2048, 8192, False),    # above two rows
    (1, 3584, 4608, False),    # Qwen2-7B: 14 > 0.6 x 20 k-blocks per CTA
    (1, 4096, 6144, False),    # Llama-3-8B: 22 > 0.6 x 26
    (1, 8192, 10240, False),   # Llama-3-70B: 76 > 0.6 x 86
    (1, 4096, 28672, False),   # gate/up: the same configuration
    (1, 4096, 512, False),     # the library would not run the cluster kernel
])
def test_grid_rule(fake_library, M, H, N, expect):
    assert fk._grid_preferred(M, H, N, _lib.BF16, 0) is expect


def test_kblocks_per_cta():
    assert fk._kblocks_per_cta(info(_lib.SCHED_DECODE, 2, 5, 120), 4096) == 26   # 2 x ceil(64 / 5)
    assert fk._kblocks_per_cta(info(_lib.SCHED_GRID, 1, 4, 144), 3584) == 14     # 1 x ceil(56 / 4)
    assert fk._kblocks_per_cta(info(_lib.SCHED_GRID, 1, 3, 144), 4104) == 22     # ragged K: ceil(65 / 3)


def test_alignment_gate():
    """The grid schedule is only taken for tensors the tensor-core schedules accept."""
    import torch

    a = torch.zeros(64, dtype=torch.bfloat16)
    assert fk._tma_ready(4096, [a], [4096, 4096])
    assert not fk._tma_ready(4100, [a], [4100])          # H % 8 != 0
    assert not fk._tma_ready(4096, [a], [4096, 4100])    # a row stride not a multiple of 8
    assert not fk._tma_ready(4096, [a[1:]], [4096])      # data pointer not 16-byte aligned
