"""The C-ABI library: it loads, exports every entry point include/*.h declares, and
rejects invalid arguments with the documented codes before touching CUDA.  CPU only
(no kernel is launched: every call here fails validation first)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from triton_fused_rmsnorm_qkv import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_symbols() -> set[str]:
    names = set()
    for h in HEADERS:
        for m in re.finditer(r"FQKV_API\s+[\w\s\*]+?\b(fqkv_\w+)\s*\(", h.read_text()):
            names.add(m.group(1))
    return names


def test_header_declares_the_abi():
    assert declared_symbols() == set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert _lib.version() == 102


FAKE = 0x100000  # 16-byte aligned, never dereferenced: validation fails before any launch


def call(**kw):
    a = dict(x=FAKE, r=FAKE * 2, g=FAKE * 3, gdt=_lib.BF16, w=FAKE * 4, out=FAKE * 64, rout=None,
             M=4, H=256, N=512, ldx=256, ldr=256, ldw=256, ldo=512, ldro=256, eps=1e-5, dtype=_lib.BF16,
             schedule=_lib.SCHED_AUTO, flags=0, ws=None, ws_bytes=0, stream=None)
    a.update(kw)
    # Keep fake buffers far apart so only the aliasing tests alias.
    return _lib.launch(a["x"], a["r"], a["g"], a["gdt"], a["w"], a["out"], a["rout"], a["M"], a["H"], a["N"],
                       a["ldx"], a["ldr"], a["ldw"], a["ldo"], a["ldro"], a["eps"], a["dtype"], a["schedule"],
                       a["flags"], a["ws"], a["ws_bytes"], a["stream"])


SPACED = dict(x=1 << 32, r=2 << 32, g=3 << 32, w=4 << 32, out=5 << 32)


@pytest.mark.parametrize("kw,code", [
    (dict(x=None), _lib.ERR_NULL),
    (dict(g=None), _lib.ERR_NULL),
    (dict(w=None), _lib.ERR_NULL),
    (dict(out=None), _lib.ERR_NULL),
    (dict(dtype=2), _lib.ERR_DTYPE),
    (dict(dtype=7), _lib.ERR_DTYPE),
    (dict(gdt=5), _lib.ERR_DTYPE),
    (dict(M=0), _lib.ERR_SHAPE),
    (dict(H=0), _lib.ERR_SHAPE),
    (dict(N=-3), _lib.ERR_SHAPE),
    (dict(ldx=100), _lib.ERR_SHAPE),
    (dict(ldw=255), _lib.ERR_SHAPE),
    (dict(ldo=511), _lib.ERR_SHAPE),
    (dict(ldr=128), _lib.ERR_SHAPE),
    (dict(M=1 << 31), _lib.ERR_SHAPE),
    (dict(schedule=9), _lib.ERR_SCHEDULE),
    (dict(flags=64), _lib.ERR_SCHEDULE),
    # the failure-path test flag is for the fused decode kernels only
    (dict(schedule=_lib.SCHED_SPLIT, flags=_lib.FLAG_TEST_WITHHOLD), _lib.ERR_SCHEDULE),
    (dict(schedule=_lib.SCHED_PREFILL, M=4096, flags=_lib.FLAG_TEST_WITHHOLD), _lib.ERR_SCHEDULE),
    (dict(schedule=_lib.SCHED_SIMT, flags=_lib.FLAG_TEST_WITHHOLD), _lib.ERR_SCHEDULE),
    (dict(H=260, ldx=260, ldr=260, ldw=260, flags=_lib.FLAG_TEST_WITHHOLD), _lib.ERR_SCHEDULE),
    (dict(schedule=_lib.SCHED_DECODE, M=65), _lib.ERR_SCHEDULE),
    (dict(schedule=_lib.SCHED_SPLIT, M=129), _lib.ERR_SCHEDULE),
    (dict(schedule=_lib.SCHED_GRID, M=9), _lib.ERR_SCHEDULE),
    (dict(schedule=_lib.SCHED_GRID, M=1, N=131200, ldo=131200), _lib.ERR_SCHEDULE),
    (dict(schedule=5), _lib.ERR_SCHEDULE),
    (dict(schedule=_lib.SCHED_GRID, M=1, ws=None), _lib.ERR_WORKSPACE),
    (dict(schedule=_lib.SCHED_GRID, M=1, ws=(6 << 32) + 16, ws_bytes=1 << 30), _lib.ERR_ALIGN),
    (dict(schedule=_lib.SCHED_GRID, M=1, x=(1 << 32) + 2), _lib.ERR_ALIGN),
    (dict(schedule=_lib.SCHED_DECODE, H=260, ldx=260, ldr=260, ldw=260, ldro=260), _lib.ERR_ALIGN),
    (dict(schedule=_lib.SCHED_DECODE, x=(1 << 32) + 2), _lib.ERR_ALIGN),
    (dict(schedule=_lib.SCHED_PREFILL, M=4096, ws=None), _lib.ERR_WORKSPACE),
    (dict(schedule=_lib.SCHED_PREFILL, M=4096, ws=6 << 32, ws_bytes=1024), _lib.ERR_WORKSPACE),
    (dict(schedule=_lib.SCHED_PREFILL, M=4096, ws=(6 << 32) + 16, ws_bytes=1 << 30), _lib.ERR_ALIGN),
    (dict(out=(1 << 32) + 64), _lib.ERR_ALIAS),
    (dict(rout=(2 << 32) + 64), _lib.ERR_ALIAS),
])
def test_invalid_arguments_are_rejected(kw, code):
    args = dict(SPACED)
    args.update(kw)
    assert call(**args) == code
    assert _lib.last_error() != ""


def test_python_error_mapping():
    with pytest.raises(TypeError):
        _lib.check(_lib.ERR_DTYPE)
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_SHAPE)
    with pytest.raises(RuntimeError):
        _lib.check(-1)


def _split_bytes(M, H, N):
    """Normalised rows + stream-K partial slots (320 CTAs x 2 x MPAD x 128 fp32) + counters."""
    a = lambda b: (b + 255) // 256 * 256  # noqa: E731
    mpad = 16 if M <= 16 else 32 if M <= 32 else 64 if M <= 64 else 128
    return a(M * H * 2) + a(320 * 2 * mpad * 128 * 4) + a(((N + 127) // 128) * 4)


@pytest.mark.parametrize("M,H,sched,expect", [
    (1, 4096, _lib.SCHED_AUTO, 0),                  # fused decode: no scratch
    (16, 4096, _lib.SCHED_DECODE, 0),
    (64, 4096, _lib.SCHED_AUTO, 0),                 # fused decode up to M = 64
    (65, 4096, _lib.SCHED_AUTO, (65 * 4096 * 2 + 255) // 256 * 256),   # prefill: pre-pass scratch
    (16, 4096, _lib.SCHED_SPLIT, _split_bytes(16, 4096, 6144)),
    (2048, 4096, _lib.SCHED_PREFILL, 2048 * 4096 * 2),           # pre-pass scratch only
    (7, 4100, _lib.SCHED_AUTO, 0),                  # H % 8 != 0 -> SIMT, no scratch
    # grid decode: 4096 bytes of counters + up to 8 partial slots per (48 + 5) tiles x M rows
    (1, 4096, _lib.SCHED_GRID, 4096 + 8 * 53 * 128 * 1 * 4),
    (8, 4096, _lib.SCHED_GRID, 4096 + 8 * 53 * 128 * 8 * 4),
    (3, 100, _lib.SCHED_SIMT, 0),
])
def test_workspace_sizes(M, H, sched, expect):
    assert _lib.workspace_bytes(M, H, 6144, _lib.BF16, sched) == expect


def test_workspace_size_rejects_bad_arguments():
    with pytest.raises(ValueError):
        _lib.workspace_bytes(0, 4096, 6144, _lib.BF16, -1)
    with pytest.raises(TypeError):
        _lib.workspace_bytes(4, 4096, 6144, 9, -1)


def rope_call(**kw):
    a = dict(qkv=1 << 32, ldq=6144, cos=2 << 32, sin=3 << 32, cb=1, q=4 << 32, k=5 << 32, v=6 << 32, B=2, S=3,
             nq=32, nkv=8, d=128, dtype=_lib.BF16, stream=None)
    a.update(kw)
    return _lib.rope_split(a["qkv"], a["ldq"], a["cos"], a["sin"], a["cb"], a["q"], a["k"], a["v"], a["B"], a["S"],
                           a["nq"], a["nkv"], a["d"], a["dtype"], a["stream"])


@pytest.mark.parametrize("kw,code", [
    (dict(qkv=None), _lib.ERR_NULL),
    (dict(sin=None), _lib.ERR_NULL),
    (dict(v=None), _lib.ERR_NULL),
    (dict(dtype=_lib.F32), _lib.ERR_DTYPE),
    (dict(B=0), _lib.ERR_SHAPE),
    (dict(nkv=0), _lib.ERR_SHAPE),
    (dict(d=120), _lib.ERR_SHAPE),           # head_dim must be a multiple of 16
    (dict(ldq=6143), _lib.ERR_SHAPE),        # row shorter than (n_q + 2 n_kv) d
    (dict(cb=3), _lib.ERR_SHAPE),            # cos / sin hold 1 or B batch rows
    (dict(ldq=6148), _lib.ERR_ALIGN),        # row stride not a multiple of 8 elements
    (dict(q=(4 << 32) + 8), _lib.ERR_ALIGN),
    (dict(q=(1 << 32) + 64), _lib.ERR_ALIAS),  # q inside qkv
    (dict(k=(4 << 32) + 4096), _lib.ERR_ALIAS),  # k inside q
])
def test_rope_split_rejects_before_any_cuda_call(kw, code):
    """fqkv_rope_split validates its arguments before touching the device."""
    assert rope_call(**kw) == code, _lib.last_error()


def fp8_call(**kw):
    a = dict(x=1 << 32, r=2 << 32, g=3 << 32, gdt=_lib.BF16, w=4 << 32, sc=5 << 32, out=6 << 32, rout=None,
             M=4, H=256, N=512, ldx=256, ldr=256, ldw=256, ldo=512, ldro=256, eps=1e-5, dtype=_lib.BF16, flags=0,
             stream=None)
    a.update(kw)
    return _lib.launch_fp8w(a["x"], a["r"], a["g"], a["gdt"], a["w"], a["sc"], a["out"], a["rout"], a["M"], a["H"],
                            a["N"], a["ldx"], a["ldr"], a["ldw"], a["ldo"], a["ldro"], a["eps"], a["dtype"], a["flags"],
                            a["stream"])


@pytest.mark.parametrize("kw,code", [
    (dict(w=None), _lib.ERR_NULL),
    (dict(sc=None), _lib.ERR_NULL),
    (dict(flags=_lib.FLAG_TEST_WITHHOLD), _lib.ERR_SCHEDULE),
    (dict(x=None), _lib.ERR_NULL),
    (dict(dtype=_lib.F32), _lib.ERR_DTYPE),
    (dict(M=65), _lib.ERR_SCHEDULE),          # decode sizes only
    (dict(ldw=255), _lib.ERR_SHAPE),
    (dict(ldw=264), _lib.ERR_ALIGN),          # row pitch not a multiple of 16 bytes
    (dict(w=(4 << 32) + 8), _lib.ERR_ALIGN),
    (dict(sc=(5 << 32) + 2), _lib.ERR_ALIGN),
    (dict(out=(4 << 32) + 1024), _lib.ERR_ALIAS),   # out inside the weight
])
def test_fp8w_rejects_before_any_cuda_call(kw, code):
    assert fp8_call(**kw) == code, _lib.last_error()


def test_profile_case_parses_its_arguments():
    """The profiler workload (``bench.py --profile-case``) takes its shape and schedule from
    the command line (no GPU needed to print its usage)."""
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    res = subprocess.run([sys.executable, str(root / "bench.py"), "--help"], capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr
    for opt in ("--profile-case", "--H", "--N", "--schedule", "--fp8w", "--calls"):
        assert opt in res.stdout


def fused_rope_call(**kw):
    a = dict(x=1 << 32, r=2 << 32, g=3 << 32, gdt=_lib.BF16, w=4 << 32, q=5 << 32, k=6 << 32, v=7 << 32,
             rout=None, B=1, S=1, H=4096, ldx=4096, ldr=4096, ldw=4096, ldro=4096, cos=8 << 32, sin=9 << 32,
             cb=1, n_q=32, n_kv=8, d=128, eps=1e-5, dtype=_lib.BF16, flags=0, stream=None)
    a.update(kw)
    return _lib.launch_rope(a["x"], a["r"], a["g"], a["gdt"], a["w"], a["q"], a["k"], a["v"], a["rout"], a["B"],
                            a["S"], a["H"], a["ldx"], a["ldr"], a["ldw"], a["ldro"], a["cos"], a["sin"], a["cb"],
                            a["n_q"], a["n_kv"], a["d"], a["eps"], a["dtype"], a["flags"], a["stream"])


@pytest.mark.parametrize("kw,code", [
    (dict(q=None), _lib.ERR_NULL),
    (dict(cos=None), _lib.ERR_NULL),
    (dict(dtype=_lib.F32), _lib.ERR_DTYPE),
    (dict(d=96), _lib.ERR_SHAPE),                     # the epilogue takes head_dim 64 or 128
    (dict(cb=3, B=2), _lib.ERR_SHAPE),                # cos rows neither 1 nor B
    (dict(B=33), _lib.ERR_SCHEDULE),                  # more tokens than the decode epilogue takes
    (dict(flags=_lib.FLAG_TEST_WITHHOLD), _lib.ERR_SCHEDULE),
    (dict(ldw=4000), _lib.ERR_SHAPE),
    (dict(q=(1 << 32) + 256), _lib.ERR_ALIAS),        # q inside x
    (dict(k=(5 << 32) + 256), _lib.ERR_ALIAS),        # k inside q
    (dict(cos=(8 << 32) + 2), _lib.ERR_ALIGN),
])
def test_fused_rope_rejects_before_any_cuda_call(kw, code):
    assert fused_rope_call(**kw) == code, _lib.last_error()
