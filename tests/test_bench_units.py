"""The benchmark's algorithmic units, on the CPU.

``bench.algorithmic_bytes`` is the numerator of every roofline figure the benchmark
reports: e * (N*H + H + M*H + R*M*H + M*N + R*M*H) for weight, gain, x, residual, output and
the returned updated residual.  Pinned here to the byte counts of the configurations it is
quoted on, and the workload table to the model shapes.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


@pytest.mark.parametrize("M,H,N,res,expect", [
    (1, 4096, 6144, True, 50_376_704),     # Llama-3-8B decode
    (4, 4096, 6144, True, 50_487_296),
    (16, 4096, 6144, True, 50_929_664),
    (64, 4096, 6144, True, 52_699_136),
    (1, 3584, 4608, False, 33_053_696),    # Qwen2-7B decode, no residual
    (16, 3584, 4608, False, 33_299_456),
    (64, 3584, 4608, False, 34_085_888),
    (1, 3584, 4608, True, 33_068_032),     # Qwen2-7B decode, residual added and returned
    (16, 3584, 4608, True, 33_528_832),
    (64, 3584, 4608, True, 35_003_392),
])
def test_algorithmic_bytes(M, H, N, res, expect):
    assert bench.algorithmic_bytes(M, H, N, res) == expect


def test_workload_shapes():
    n_out = {name: (w["n_q"] + 2 * w["n_kv"]) * w["d"] for name, w in bench.WORKLOADS.items()}
    assert n_out["llama3-8b-decode"] == 6144 and bench.WORKLOADS["llama3-8b-decode"]["H"] == 4096
    assert n_out["qwen2-7b-decode"] == 4608 and bench.WORKLOADS["qwen2-7b-decode"]["H"] == 3584
    assert n_out["llama3-70b"] == 10240 and bench.WORKLOADS["llama3-70b"]["H"] == 8192
    assert n_out["llama3-8b-mlp"] == 2 * 14336
    assert bench.WORKLOADS["llama3-8b-decode"]["M"] == 16 and bench.WORKLOADS["llama3-8b-decode"]["sets"] == 32
