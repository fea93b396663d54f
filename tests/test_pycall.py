"""The CPython fast path for fqkv_launch (csrc/fqkv_pycall.c) against the ctypes binding:
for arguments the library rejects before any CUDA call, both paths return the same code
and leave the same error text; malformed argument lists raise in Python."""
from __future__ import annotations

import pytest

from triton_fused_rmsnorm_qkv import _lib

BF16 = _lib.BF16
# (x, r, g, gdt, w, out, rout, M, H, N, ldx, ldr, ldw, ldo, ldro, eps, dtype, schedule, flags, ws, ws_bytes, stream)
P = 1 << 20  # a 16-byte-aligned fake device address (never dereferenced: validation fails first)
CASES = [
    (None, None, None, BF16, None, None, None, 16, 4096, 6144, 4096, 4096, 4096, 6144, 4096, 1e-5, BF16, -1, 1, None, 0, 0),
    (P, None, P, BF16, P, P, None, 0, 4096, 6144, 4096, 0, 4096, 6144, 0, 1e-5, BF16, -1, 1, None, 0, 0),
    (P, None, P, BF16, P, P, None, 16, 4096, 6144, 4096, 0, 4096, 6144, 0, 1e-5, 7, -1, 1, None, 0, 0),
    (P, None, P, BF16, P, P, None, 16, 4096, 6144, 100, 0, 4096, 6144, 0, 1e-5, BF16, -1, 1, None, 0, 0),
    (P, None, P, BF16, P, P, None, 16, 4096, 6144, 4096, 0, 4096, 6144, 0, 1e-5, BF16, 99, 1, None, 0, 0),
    (P + 2, None, P, BF16, P * 2, P * 4, None, 16, 4096, 6144, 4096, 0, 4096, 6144, 0, 1e-5, BF16, 1, 1, None, 0, 0),
]


def _via_ctypes(args):
    saved, _lib._pycall = _lib._pycall, None
    try:
        return _lib.launch(*args), _lib.last_error()
    finally:
        _lib._pycall = saved


@pytest.mark.skipif(_lib._pycall is None, reason="the CPython fast path is not built")
@pytest.mark.parametrize("args", CASES)
def test_fast_path_matches_ctypes(args):
    _lib.load()
    rc_c, err_c = _via_ctypes(args)
    rc_f, err_f = _lib.launch(*args), _lib.last_error()
    assert rc_c > 0 and (rc_f, err_f) == (rc_c, err_c)


@pytest.mark.skipif(_lib._pycall is None, reason="the CPython fast path is not built")
def test_fast_path_rejects_malformed_argument_lists():
    _lib.load()
    with pytest.raises(TypeError):
        _lib._pycall.launch(*CASES[0][:-1])
    with pytest.raises(TypeError):
        _lib._pycall.launch(*(CASES[1][:15] + ("eps",) + CASES[1][16:]))
