"""Fused residual add + RMSNorm + packed projection on B200 (sm_100a).

Drop-in for the reference's ``src/triton_fused_rmsnorm_qkv/kernel.py``: the same public
functions with the same arguments, return values and assertion errors, backed by
hand-written sm_100a CUDA kernels in ``libfqkv.so`` instead of Triton.

    hidden = x + residual                          (or x when residual is None)
    normed = dtype((fp32(hidden) * rstd) * fp32(rms_weight)),  rstd = 1/sqrt(mean(hidden^2) + eps)
    out    = normed @ weight^T                     (fp32 accumulation, output in x.dtype)

Where the reference dispatches between two Triton kernels at M = 32 rows
(kernel.py:360, :406) and picks tiles by autotuning (kernel.py:122-128, :264-268), the
library chooses one of its kernel families from (M, H, N, SM count):

* ``decode``  (M <= 64): one fused kernel -- swap-AB tcgen05 MMA, the weight streamed
  by TMA, K split across a thread-block cluster whose CTAs exchange row sums of
  squares and partial tiles through distributed shared memory.
* ``grid``    (M <= 8): the same fused kernel without clusters, so that its CTAs cover
  nearly every SM.  Each CTA reads the whole activation rows, and the CTA that finishes a
  tile last sums the partial tiles through a zero-filled workspace this module keeps per
  device and stream.  Chosen automatically for M <= ``_GRID_AUTO_MAX_M`` only when it cuts
  the weight bytes per CTA far below the cluster kernel's (``_grid_preferred``); no measured
  model shape qualifies, so in practice it runs when forced (``schedule="grid"``).
* ``split``   (M <= 64 when no decode configuration fits the device, or when forced; up
  to M = 128): norm pre-pass + a stream-K swap-AB GEMM reading the normalised rows by TMA.
* ``prefill`` (M > 64): norm pre-pass + persistent 128 x BN tcgen05 GEMM.
* ``simt``    any shape/stride the TMA paths cannot take (H % 8 != 0, unaligned data).

Extensions (keyword-only, so the reference call sites keep working): ``residual_out``
receives the updated residual ``x + residual`` (bit-exact in the working dtype),
``schedule`` forces a kernel family, ``static_weights`` lets the decode kernel start
streaming the weight before the preceding kernel in the stream has finished.
"""
from __future__ import annotations

import collections
import contextlib
import os
from typing import Optional, Tuple

import torch

from . import _lib

# The reference switches kernels at M = 32 (kernel.py:360).  The B200 dispatch lives in
# the C library; these mirror its bounds for readers of the Python API.
_PERSISTENT_THRESHOLD = 32
_DTYPE_CODE = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}
_GAIN_CODE = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}

# (M, H) -> N of the last call, so get_autotune_best_config(M, H) can describe the
# schedule the library chose for it (the reference reads Triton's autotune cache).
_seen_shapes: dict[tuple[int, int], int] = {}

# Workspace bytes per (M, H, N, dtype, schedule, device): the library's answer depends only
# on these, and asking it every call costs a round trip through ctypes.
_ws_bytes: dict[tuple, int] = {}

# The automatic choice of the grid schedule: at most this many rows (every CTA reads whole
# rows, which stops paying beyond a few), and at most this fraction of the cluster kernel's
# weight bytes per CTA.  Since the cluster kernel spreads the norm phase of one to four rows
# over all its norm warps, it beats the grid variant on every measured shape (B200,
# graph-timed, M = 1 / 2, cluster against grid, us): Qwen2-7B 10.50 / 10.91 against 11.60 /
# 12.23 (bytes fraction 0.74; since then the cluster kernel's two-tile stages take it to
# 9.41 / 10.52 at M = 1 / 16), Llama-3-8B 11.69 / 11.63 against 14.32 / 14.94 (0.85),
# Llama-3-70B 30.64 / 31.16 against 33.18 / 35.77 (0.88).  The fraction is therefore set
# below all of them: the grid schedule is taken automatically only where it would stream at
# most 0.6 of the cluster kernel's bytes per CTA.
_GRID_AUTO_MAX_M = 2
_GRID_AUTO_MAX_BYTES = 0.6
# (M, H, N, dtype, device) -> whether the automatic choice is the grid schedule.
_grid_choice: dict[tuple, bool] = {}
# Workspaces kept between calls.  Launches on one stream run in order, so calls on a
# stream can share one buffer:
#  * (device, stream) -> zero-filled workspace of the grid schedule for eager calls.  Its
#    launches leave the arrival counters at zero, so the buffer is zeroed once.
#  * (device, stream, capture id) -> the same for calls made while that stream is being
#    captured into a CUDA graph.  It is created (zero-filled) inside the capture, so every
#    replay of that graph zeroes it before its first grid launch, and no other graph and no
#    eager call uses it: graphs replayed at the same time on different streams do not share
#    counters.  The newest _CAPTURE_KEEP captures keep theirs.
#  * (device, stream) -> workspace of the pre-pass schedules (split, prefill) for eager
#    calls; nothing in it needs to start at zero.  Calls made during a capture allocate
#    theirs from the graph's private pool instead.
_grid_ws: dict[tuple[int, int], torch.Tensor] = {}
_grid_ws_capture: "collections.OrderedDict[tuple[int, int, int], torch.Tensor]" = collections.OrderedDict()
_CAPTURE_KEEP = 16
_prepass_ws: dict[tuple[int, int], torch.Tensor] = {}


def _env_flag(name: str) -> bool:
    return os.environ.get(name, "") not in ("", "0", "false", "False")


def _schedule_code(schedule) -> int:
    if schedule is None:
        forced = os.environ.get("FQKV_FORCE_SCHEDULE", "")
        return _lib.SCHEDULE_BY_NAME[forced] if forced else _lib.SCHED_AUTO
    if isinstance(schedule, str):
        if schedule not in _lib.SCHEDULE_BY_NAME:
            raise ValueError(f"unknown schedule {schedule!r}; expected one of {sorted(_lib.SCHEDULE_BY_NAME)}")
        return _lib.SCHEDULE_BY_NAME[schedule]
    return int(schedule)


def _current_device() -> int:
    """Index of the current CUDA device (without torch.cuda's lazy-initialisation checks)."""
    raw = getattr(torch._C, "_cuda_getDevice", None)
    return raw() if raw is not None else torch.cuda.current_device()


def _current_stream(index: int) -> int:
    """Handle of the current CUDA stream of device ``index`` (without building a Stream object)."""
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    return raw(index) if raw is not None else torch.cuda.current_stream(index).cuda_stream


def _rows(t: torch.Tensor, M: int, H: int) -> torch.Tensor:
    """``t`` (B, S, H) as M = B*S rows with one row stride and unit column stride.

    The tensor is returned as it is when its rows already are uniformly strided (the
    common case: no view is created); otherwise as an [M, H] view, or a copy if even that
    is not possible."""
    if t.dim() == 3 and t.stride(2) == 1 and (t.shape[0] == 1 or t.stride(0) == t.shape[1] * t.stride(1)):
        return t
    t2 = t.reshape(M, H)
    if t2.stride(1) != 1:
        t2 = t2.contiguous()
    return t2


def _row_stride(t: torch.Tensor) -> int:
    return t.stride(-2) if t.dim() >= 2 else t.shape[-1]


def _kblocks_per_cta(info: dict, H: int) -> int:
    """Weight k-blocks (128 rows x 64) one CTA of a decode configuration streams."""
    kb = (H + 63) // 64
    return info["block_n"] // 128 * -(-kb // info["split_k"])


def _grid_preferred(M: int, H: int, N: int, dtype_code: int, index: int) -> bool:
    """Whether the automatic schedule for this shape is ``grid``: at most
    ``_GRID_AUTO_MAX_M`` rows, the library would pick the cluster decode kernel, and the
    grid configuration streams at most ``_GRID_AUTO_MAX_BYTES`` of its weight bytes per CTA."""
    key = (M, H, N, dtype_code, index)
    hit = _grid_choice.get(key)
    if hit is None:
        hit = False
        if M <= _GRID_AUTO_MAX_M:
            auto = _lib.query_schedule(M, H, N, dtype_code, _lib.SCHED_AUTO)
            if auto["schedule"] == _lib.SCHED_DECODE:
                try:
                    grid = _lib.query_schedule(M, H, N, dtype_code, _lib.SCHED_GRID)
                except (RuntimeError, ValueError, TypeError):
                    grid = None
                hit = grid is not None and (
                    _kblocks_per_cta(grid, H) <= _GRID_AUTO_MAX_BYTES * _kblocks_per_cta(auto, H))
        _grid_choice[key] = hit
    return hit


def _tma_ready(H: int, tensors, strides) -> bool:
    """The alignment the library's tensor-core schedules need (else it runs ``simt``)."""
    return (H % 8 == 0 and H <= 16384 and all(t.data_ptr() % 16 == 0 for t in tensors)
            and all(s % 8 == 0 for s in strides))


def _grid_workspace(index: int, stream: int, nbytes: int, dev: torch.device) -> torch.Tensor:
    """The zero-filled grid-schedule workspace of this device and stream (and of the capture
    running on it, if any), grown as needed."""
    if torch.cuda.is_current_stream_capturing():
        key = (index, stream, _lib.stream_capture_id(stream))
        buf = _grid_ws_capture.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)  # a memset node of this graph
            _grid_ws_capture[key] = buf
            while len(_grid_ws_capture) > _CAPTURE_KEEP:
                _grid_ws_capture.popitem(last=False)
        return buf
    buf = _grid_ws.get((index, stream))
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _grid_ws[(index, stream)] = buf
    return buf


def _prepass_workspace(index: int, stream: int, nbytes: int, dev: torch.device) -> torch.Tensor:
    """Workspace of the pre-pass schedules: one buffer per device and stream for eager calls,
    grown as needed; a fresh one from the graph's pool while the stream is captured."""
    if torch.cuda.is_current_stream_capturing():
        return torch.empty(nbytes, dtype=torch.uint8, device=dev)
    buf = _prepass_ws.get((index, stream))
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        _prepass_ws[(index, stream)] = buf
    return buf


def _launch(x2: torch.Tensor, r2: Optional[torch.Tensor], rms_weight: torch.Tensor, weight: torch.Tensor,
            out2: torch.Tensor, rout2: Optional[torch.Tensor], eps: float, schedule: int,
            static_weights: bool, M: int) -> None:
    """Validate tensor metadata and call ``fqkv_launch`` on the current stream.  The
    activation, output and residual-out tensors are M rows of H (N) elements with one row
    stride each (see ``_rows``).  Every call goes through here, so it reads each piece of
    metadata once."""
    H = x2.shape[-1]
    N = weight.shape[0]
    xdt = x2.dtype
    dt = _DTYPE_CODE.get(xdt)
    if dt is None:
        raise TypeError(f"x must be float16 or bfloat16, got {xdt}")
    if weight.dtype != xdt:
        raise TypeError(f"weight dtype {weight.dtype} does not match x dtype {xdt}")
    if r2 is not None and r2.dtype != xdt:
        raise TypeError(f"residual dtype {r2.dtype} does not match x dtype {xdt}")
    gcode = _GAIN_CODE.get(rms_weight.dtype)
    if gcode is None:
        raise TypeError(f"rms_weight must be float32, float16 or bfloat16, got {rms_weight.dtype}")
    if rms_weight.numel() != H:
        raise ValueError(f"rms_weight must have H={H} elements, got shape {tuple(rms_weight.shape)}")
    index = x2.get_device()
    for name, t in (("residual", r2), ("rms_weight", rms_weight), ("weight", weight)):
        if t is not None and t.get_device() != index:
            raise ValueError(f"{name} is on {t.device}, x is on {x2.device}")
    g = rms_weight if rms_weight.dim() == 1 else rms_weight.reshape(H)
    if g.stride(0) != 1:
        g = g.contiguous()
    w = weight if weight.stride(1) == 1 else weight.contiguous()
    code = _schedule_code(schedule)
    flags = _lib.FLAG_PDL | (_lib.FLAG_STATIC_WEIGHTS if static_weights else 0)
    ldx, ldw, ldo = _row_stride(x2), w.stride(0), _row_stride(out2)
    ldr = _row_stride(r2) if r2 is not None else 0
    ldro = _row_stride(rout2) if rout2 is not None else 0
    if index == _current_device():
        rc = _call(x2, r2, g, gcode, w, out2, rout2, M, H, N, ldx, ldr, ldw, ldo, ldro, eps, dt, code, flags, index)
    else:
        with torch.cuda.device(index):
            rc = _call(x2, r2, g, gcode, w, out2, rout2, M, H, N, ldx, ldr, ldw, ldo, ldro, eps, dt, code, flags,
                       index)
    _lib.check(rc)
    _seen_shapes[(M, H)] = N


def _call(x2, r2, g, gcode, w, out2, rout2, M, H, N, ldx, ldr, ldw, ldo, ldro, eps, dt, code, flags, index) -> int:
    """Choose the workspace (and the grid schedule where it applies) and call ``fqkv_launch``
    with device ``index`` current."""
    if code == _lib.SCHED_AUTO and M <= _GRID_AUTO_MAX_M and _grid_preferred(M, H, N, dt, index):
        tensors = [t for t in (x2, r2, g, w, rout2) if t is not None]
        strides = [ldx, ldw] + ([ldr] if r2 is not None else []) + ([ldro] if rout2 is not None else [])
        if _tma_ready(H, tensors, strides):
            code = _lib.SCHED_GRID
    key = (M, H, N, dt, code, index)
    ws_bytes = _ws_bytes.get(key)
    if ws_bytes is None:
        ws_bytes = _ws_bytes[key] = _lib.workspace_bytes(M, H, N, dt, code)
    stream = _current_stream(index)
    if code == _lib.SCHED_GRID:
        ws = _grid_workspace(index, stream, ws_bytes, x2.device)
    else:
        ws = _prepass_workspace(index, stream, ws_bytes, x2.device) if ws_bytes > 0 else None
    return _lib.launch(
        x2.data_ptr(), r2.data_ptr() if r2 is not None else None, g.data_ptr(), gcode, w.data_ptr(),
        out2.data_ptr(), rout2.data_ptr() if rout2 is not None else None, M, H, N, ldx, ldr, ldw, ldo, ldro,
        float(eps), dt, code, flags, ws.data_ptr() if ws is not None else None, ws_bytes, stream)


def _fused(x, residual, rms_weight, weight, eps, *, residual_out, schedule, static_weights, out=None):
    assert x.is_cuda, "Fused kernel requires CUDA tensors"
    B, S, H = x.shape
    N_OUT = weight.shape[0]
    assert weight.shape[1] == H, f"weight must be (N_OUT, H); got {weight.shape} for H={H}"
    M = B * S
    x2 = _rows(x, M, H)
    r2 = None
    if residual is not None:
        if residual.numel() != M * H:
            raise ValueError(f"residual must match x {tuple(x.shape)}, got {tuple(residual.shape)}")
        r2 = _rows(residual, M, H)
    if out is None:
        out = torch.empty(B, S, N_OUT, dtype=x.dtype, device=x.device)
    elif (out.shape != (B, S, N_OUT) or out.dtype != x.dtype or out.get_device() != x.get_device()
          or out.stride(2) != 1 or (B > 1 and out.stride(0) != S * out.stride(1))):
        raise ValueError(f"out must be a ({B}, {S}, {N_OUT}) {x.dtype} tensor on {x.device} whose rows are "
                         "uniformly strided with unit stride along N")
    rout2 = None
    if residual_out is not None:
        if residual_out.numel() != M * H or residual_out.dtype != x.dtype or residual_out.get_device() != x.get_device():
            raise ValueError("residual_out must have the shape, dtype and device of x")
        rout2 = _rows(residual_out, M, H)
        if rout2.data_ptr() != residual_out.data_ptr() or rout2.stride(-1) != 1:
            raise ValueError("residual_out must be writable as M rows with unit stride along H")
    if static_weights is None:
        static_weights = _env_flag("FQKV_STATIC_WEIGHTS")
    _launch(x2, r2, rms_weight, weight, out, rout2, eps, schedule, static_weights, M)
    return out


def fused_rmsnorm_residual_matmul(
    x: torch.Tensor,
    residual: Optional[torch.Tensor],
    rms_weight: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    *,
    residual_out: Optional[torch.Tensor] = None,
    schedule=None,
    static_weights: Optional[bool] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Fused (optional residual) + RMSNorm + arbitrary-width matmul (kernel.py:363-436).

    Args:
        x: (B, S, H) activations, float16 or bfloat16.
        residual: (B, S, H) residual stream, or None to skip the add.
        rms_weight: (H,) RMSNorm gain (float32, float16 or bfloat16).
        weight: (N_OUT, H) projection, e.g. the packed GQA weight [Wq; Wk; Wv].
        eps: RMSNorm epsilon.
        residual_out: optional (B, S, H) tensor that receives x + residual.
        schedule: None/"auto", "decode", "grid", "split", "prefill" or "simt" ("naive").
        static_weights: weight is not written by the preceding kernel in the stream
            (default: environment variable FQKV_STATIC_WEIGHTS).
        out: optional (B, S, N_OUT) tensor in x.dtype that receives the result (rows
            uniformly strided, unit stride along N) instead of a new allocation.

    Returns:
        (B, S, N_OUT) tensor in x.dtype (``out`` when given).
    """
    return _fused(x, residual, rms_weight, weight, eps, residual_out=residual_out, schedule=schedule,
                  static_weights=static_weights, out=out)


def fused_add_rmsnorm_matmul(
    x: torch.Tensor,
    residual: Optional[torch.Tensor],
    rms_weight: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
    *,
    return_residual: bool = True,
    schedule=None,
    static_weights: Optional[bool] = None,
    out: Optional[torch.Tensor] = None,
    residual_out: Optional[torch.Tensor] = None,
):
    """As ``fused_rmsnorm_residual_matmul``, also returning the updated residual.

    Returns ``(out, hidden)`` with ``hidden = x + residual`` computed once in fp32 and
    rounded to x.dtype (bit-identical to ``x + residual`` in PyTorch, baseline.py:48),
    or ``out`` alone when ``return_residual`` is False.  ``out`` and ``residual_out``
    (with ``return_residual``) receive the two results instead of new allocations.
    """
    hidden = None
    if return_residual:
        hidden = residual_out if residual_out is not None else torch.empty_like(x)
    out = _fused(x, residual, rms_weight, weight, eps, residual_out=hidden, schedule=schedule,
                 static_weights=static_weights, out=out)
    return (out, hidden) if return_residual else out


def fused_rmsnorm_residual_qkv(
    x: torch.Tensor,
    residual: Optional[torch.Tensor],
    rms_weight: torch.Tensor,
    qkv_weight: torch.Tensor,
    eps: float = 1e-6,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """MHA convenience wrapper for a (3*H, H) packed weight (kernel.py:439-461).

    For GQA call ``fused_rmsnorm_residual_matmul`` with the (H + 2*H_kv, H) weight and
    split the result by the real widths.
    """
    H = x.shape[-1]
    assert qkv_weight.shape == (3 * H, H), (
        f"qkv_weight must be (3*H, H); got {qkv_weight.shape}. "
        "For GQA, call fused_rmsnorm_residual_matmul directly."
    )
    out = fused_rmsnorm_residual_matmul(x, residual, rms_weight, qkv_weight, eps)
    q, k, v = out.chunk(3, dim=-1)
    return q, k, v


E4M3_MAX = 448.0  # largest finite float8_e4m3fn value


def quantize_weight_e4m3(weight: torch.Tensor):
    """(w8, scale): ``weight`` (N, H) as float8_e4m3fn with one fp32 scale per row,
    ``scale[n] = max_k |weight[n, k]| / 448`` (1 for an all-zero row), ``w8 = weight / scale``
    rounded to e4m3.  ``w8.float() * scale[:, None]`` approximates ``weight``."""
    if weight.dim() != 2:
        raise ValueError(f"weight must be (N, H), got shape {tuple(weight.shape)}")
    w = weight.float()
    amax = w.abs().amax(dim=1)
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    w8 = (w / scale[:, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return w8.contiguous(), scale.contiguous()


def fused_add_rmsnorm_matmul_fp8w(
    x: torch.Tensor,
    residual: Optional[torch.Tensor],
    rms_weight: torch.Tensor,
    weight_e4m3: torch.Tensor,
    weight_scale: torch.Tensor,
    eps: float = 1e-6,
    *,
    return_residual: bool = True,
    static_weights: Optional[bool] = None,
):
    """``fused_add_rmsnorm_matmul`` with an FP8 (e4m3) weight and an fp32 scale per weight row.

    ``out = dtype(weight_scale[n] * sum_k normed[m, k] * weight_e4m3[n, k])`` with ``normed``
    exactly as the 16-bit path forms it (``quantize_weight_e4m3`` makes the pair from a 16-bit
    weight).  The fused decode kernel streams the one-byte weight -- half the bytes -- into
    e4m3 x e4m3 tensor-core MMAs (tcgen05 kind::f8f6f4), the normalised activations split
    exactly into e4m3 terms with a power-of-two scale per token.  Decode sizes only
    (M = B * S <= 64); larger M raise ``ValueError``.
    """
    assert x.is_cuda, "Fused kernel requires CUDA tensors"
    B, S, H = x.shape
    if weight_e4m3.dtype != torch.float8_e4m3fn:
        raise TypeError(f"weight_e4m3 must be torch.float8_e4m3fn, got {weight_e4m3.dtype}")
    N = weight_e4m3.shape[0]
    assert weight_e4m3.shape[1] == H, f"weight must be (N_OUT, H); got {weight_e4m3.shape} for H={H}"
    if weight_scale.dtype != torch.float32 or weight_scale.numel() != N:
        raise ValueError(f"weight_scale must be {N} float32 values, got {weight_scale.dtype} {tuple(weight_scale.shape)}")
    if x.dtype not in _DTYPE_CODE:
        raise TypeError(f"x must be float16 or bfloat16, got {x.dtype}")
    if rms_weight.dtype not in _GAIN_CODE or rms_weight.numel() != H:
        raise ValueError(f"rms_weight must hold H={H} float32/float16/bfloat16 values")
    for name, t in (("residual", residual), ("rms_weight", rms_weight), ("weight_e4m3", weight_e4m3),
                    ("weight_scale", weight_scale)):
        if t is not None and t.device != x.device:
            raise ValueError(f"{name} is on {t.device}, x is on {x.device}")
    M = B * S
    x2 = _rows(x, M, H)
    r2 = None
    if residual is not None:
        if residual.numel() != M * H or residual.dtype != x.dtype:
            raise ValueError(f"residual must match x {tuple(x.shape)} {x.dtype}")
        r2 = _rows(residual, M, H)
    w8 = weight_e4m3 if weight_e4m3.stride(1) == 1 else weight_e4m3.contiguous()
    sc = weight_scale.reshape(N).contiguous()
    g = rms_weight.reshape(H).contiguous()
    out = torch.empty(B, S, N, dtype=x.dtype, device=x.device)
    hidden = torch.empty_like(x) if return_residual else None
    rout2 = _rows(hidden, M, H) if hidden is not None else None
    if static_weights is None:
        static_weights = _env_flag("FQKV_STATIC_WEIGHTS")
    flags = _lib.FLAG_PDL | (_lib.FLAG_STATIC_WEIGHTS if static_weights else 0)
    dev = x.device
    ctx = contextlib.nullcontext() if dev.index == torch.cuda.current_device() else torch.cuda.device(dev)
    with ctx:
        rc = _lib.launch_fp8w(
            x2.data_ptr(), r2.data_ptr() if r2 is not None else None, g.data_ptr(), _GAIN_CODE[g.dtype],
            w8.data_ptr(), sc.data_ptr(), out.data_ptr(), rout2.data_ptr() if rout2 is not None else None,
            M, H, N, _row_stride(x2), _row_stride(r2) if r2 is not None else 0, w8.stride(0), N,
            _row_stride(rout2) if rout2 is not None else 0, float(eps), _DTYPE_CODE[x.dtype], flags,
            _current_stream(dev.index))
    _lib.check(rc, "fqkv_launch_fp8w")
    return (out, hidden) if return_residual else out


def qkv_rope_split(
    qkv: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    n_q_heads: int,
    n_kv_heads: int,
    head_dim: Optional[int] = None,
):
    """Split a packed projection output into head-major Q, K, V and rotate Q and K.

    ``qkv`` is (B, S, (n_q + 2 n_kv) * d), the output of the fused call on the packed
    ``[Wq; Wk; Wv]`` weight.  Returns ``q`` (B, n_q, S, d), ``k`` and ``v`` (B, n_kv, S, d),
    contiguous, with ``x * cos + rotate_half(x) * sin`` applied to q and k: one CUDA launch
    for what the Llama integration does with split / view / transpose and transformers'
    ``apply_rotary_pos_emb`` (llama3_patch.py:156-168), and bit-identical to it.  ``cos`` and
    ``sin`` are (B, S, d), (1, S, d) or (S, d) in qkv's dtype, as the model's rotary
    embedding returns them.
    """
    if qkv.dim() != 3:
        raise ValueError(f"qkv must be (B, S, width), got shape {tuple(qkv.shape)}")
    if qkv.dtype not in _DTYPE_CODE:
        raise TypeError(f"qkv must be float16 or bfloat16, got {qkv.dtype}")
    B, S, W = qkv.shape
    heads = n_q_heads + 2 * n_kv_heads
    if head_dim is None:
        head_dim = W // heads
    if heads * head_dim != W:
        raise ValueError(f"qkv width {W} is not ({n_q_heads} + 2 * {n_kv_heads}) * {head_dim}")
    tabs = []
    for name, t in (("cos", cos), ("sin", sin)):
        if t.dtype != qkv.dtype or t.device != qkv.device:
            raise TypeError(f"{name} must have qkv's dtype and device ({qkv.dtype}, {qkv.device})")
        if t.dim() == 2:
            t = t.unsqueeze(0)
        if t.dim() != 3 or t.shape[1:] != (S, head_dim) or t.shape[0] not in (1, B):
            raise ValueError(f"{name} must be (B, S, d), (1, S, d) or (S, d); got {tuple(t.shape)}")
        tabs.append(t.contiguous())
    if tabs[0].shape[0] != tabs[1].shape[0]:
        raise ValueError("cos and sin must have the same batch size")
    rows = _rows(qkv, B * S, W)
    q = torch.empty(B, n_q_heads, S, head_dim, dtype=qkv.dtype, device=qkv.device)
    k = torch.empty(B, n_kv_heads, S, head_dim, dtype=qkv.dtype, device=qkv.device)
    v = torch.empty_like(k)
    dev = qkv.device
    ctx = contextlib.nullcontext() if dev.index == torch.cuda.current_device() else torch.cuda.device(dev)
    with ctx:
        rc = _lib.rope_split(rows.data_ptr(), _row_stride(rows), tabs[0].data_ptr(), tabs[1].data_ptr(),
                             tabs[0].shape[0], q.data_ptr(), k.data_ptr(), v.data_ptr(), B, S, n_q_heads, n_kv_heads,
                             head_dim, _DTYPE_CODE[qkv.dtype], _current_stream(dev.index))
    _lib.check(rc, "fqkv_rope_split")
    return q, k, v


def _rope_tables(cos: torch.Tensor, sin: torch.Tensor, B: int, S: int, head_dim: int, like: torch.Tensor):
    """cos / sin as contiguous (1 or B, S, head_dim) tensors of ``like``'s dtype and device."""
    tabs = []
    for name, t in (("cos", cos), ("sin", sin)):
        if t.dtype != like.dtype or t.device != like.device:
            raise TypeError(f"{name} must have the activations' dtype and device ({like.dtype}, {like.device})")
        if t.dim() == 2:
            t = t.unsqueeze(0)
        if t.dim() != 3 or t.shape[1:] != (S, head_dim) or t.shape[0] not in (1, B):
            raise ValueError(f"{name} must be (B, S, d), (1, S, d) or (S, d); got {tuple(t.shape)}")
        tabs.append(t.contiguous())
    if tabs[0].shape[0] != tabs[1].shape[0]:
        raise ValueError("cos and sin must have the same batch size")
    return tabs


def fused_add_rmsnorm_qkv_rope(
    x: torch.Tensor,
    residual: Optional[torch.Tensor],
    rms_weight: torch.Tensor,
    qkv_weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    n_q_heads: int,
    n_kv_heads: int,
    head_dim: Optional[int] = None,
    eps: float = 1e-6,
    *,
    return_residual: bool = True,
    static_weights: Optional[bool] = None,
):
    """Residual add + RMSNorm + packed Q/K/V projection + head split + rotary embedding.

    Returns ``(q, k, v, hidden)`` (or ``(q, k, v)`` when ``return_residual`` is False):
    ``q`` (B, n_q, S, d), ``k`` and ``v`` (B, n_kv, S, d), contiguous, Q and K rotated by
    ``x * cos + rotate_half(x) * sin`` -- bit-identical to ``fused_add_rmsnorm_matmul``
    followed by ``qkv_rope_split`` (the sequence of llama3_patch.py:148-168).  Decode sizes
    (B * S <= 32, head_dim 64 or 128) run as one launch, the rotary split in the projection's
    epilogue; other sizes run the two launches.
    """
    assert x.is_cuda, "Fused kernel requires CUDA tensors"
    B, S, H = x.shape
    N = qkv_weight.shape[0]
    assert qkv_weight.shape[1] == H, f"weight must be (N_OUT, H); got {qkv_weight.shape} for H={H}"
    heads = n_q_heads + 2 * n_kv_heads
    if head_dim is None:
        head_dim = N // heads
    if heads * head_dim != N:
        raise ValueError(f"weight rows {N} are not ({n_q_heads} + 2 * {n_kv_heads}) * {head_dim}")
    dt = _DTYPE_CODE.get(x.dtype)
    if dt is None:
        raise TypeError(f"x must be float16 or bfloat16, got {x.dtype}")
    M = B * S
    hidden = torch.empty_like(x) if return_residual else None
    tabs = _rope_tables(cos, sin, B, S, head_dim, x)
    if static_weights is None:
        static_weights = _env_flag("FQKV_STATIC_WEIGHTS")
    x2 = _rows(x, M, H)
    r2 = _rows(residual, M, H) if residual is not None else None
    w = qkv_weight if qkv_weight.stride(1) == 1 else qkv_weight.contiguous()
    g = rms_weight.reshape(H)
    if g.stride(0) != 1:
        g = g.contiguous()
    gcode = _GAIN_CODE.get(g.dtype)
    tensors = [t for t in (x2, r2, g, w, hidden, *tabs) if t is not None]
    strides = [_row_stride(x2), w.stride(0)] + ([_row_stride(r2)] if r2 is not None else [])
    one_launch = (M <= 32 and head_dim in (64, 128) and gcode is not None and w.dtype == x.dtype
                  and (r2 is None or r2.dtype == x.dtype) and _tma_ready(H, tensors, strides))
    if one_launch:
        q = torch.empty(B, n_q_heads, S, head_dim, dtype=x.dtype, device=x.device)
        k = torch.empty(B, n_kv_heads, S, head_dim, dtype=x.dtype, device=x.device)
        v = torch.empty_like(k)
        rout2 = _rows(hidden, M, H) if hidden is not None else None
        flags = _lib.FLAG_PDL | (_lib.FLAG_STATIC_WEIGHTS if static_weights else 0)
        dev = x.device
        ctx = contextlib.nullcontext() if dev.index == torch.cuda.current_device() else torch.cuda.device(dev)
        with ctx:
            rc = _lib.launch_rope(
                x2.data_ptr(), r2.data_ptr() if r2 is not None else None, g.data_ptr(), gcode, w.data_ptr(),
                q.data_ptr(), k.data_ptr(), v.data_ptr(), rout2.data_ptr() if rout2 is not None else None, B, S, H,
                _row_stride(x2), _row_stride(r2) if r2 is not None else 0, w.stride(0),
                _row_stride(rout2) if rout2 is not None else 0, tabs[0].data_ptr(), tabs[1].data_ptr(),
                tabs[0].shape[0], n_q_heads, n_kv_heads, head_dim, float(eps), dt, flags, _current_stream(dev.index))
        if rc != _lib.ERR_SCHEDULE:  # no configuration fits this device: the two launches below
            _lib.check(rc, "fqkv_launch_rope")
            return (q, k, v, hidden) if return_residual else (q, k, v)
    out = _fused(x, residual, rms_weight, qkv_weight, eps, residual_out=hidden, schedule=None,
                 static_weights=static_weights)
    q, k, v = qkv_rope_split(out, tabs[0], tabs[1], n_q_heads, n_kv_heads, head_dim)
    return (q, k, v, hidden) if return_residual else (q, k, v)


def fused_rmsnorm_residual_matmul_fixed(
    x: torch.Tensor,
    residual: Optional[torch.Tensor],
    rms_weight: torch.Tensor,
    weight: torch.Tensor,
    eps: float = 1e-6,
) -> torch.Tensor:
    """Same contract with the adaptive dispatch switched off (kernel.py:469-540).

    The reference pins one untuned Triton tile for its autotune ablation; here every
    shape runs the fixed-tile CUDA-core ("simt") kernel.
    """
    assert x.is_cuda
    B, S, H = x.shape
    assert weight.shape[1] == H
    return _fused(x, residual, rms_weight, weight, eps, residual_out=None, schedule=_lib.SCHED_SIMT,
                  static_weights=False)


def fused_rmsnorm_residual_qkv_fixed(
    x: torch.Tensor,
    residual: Optional[torch.Tensor],
    rms_weight: torch.Tensor,
    qkv_weight: torch.Tensor,
    eps: float = 1e-6,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Same interface as ``fused_rmsnorm_residual_qkv`` with the dispatch off (kernel.py:543-555)."""
    H = x.shape[-1]
    assert qkv_weight.shape == (3 * H, H)
    out = fused_rmsnorm_residual_matmul_fixed(x, residual, rms_weight, qkv_weight, eps)
    q, k, v = out.chunk(3, dim=-1)
    return q, k, v


def schedule_info(M: int, H: int, N: int, dtype: torch.dtype = torch.bfloat16) -> dict:
    """The library's record (``fqkv_query_schedule``) of the schedule an automatically
    scheduled call of this shape runs on the current device, with 16-byte-aligned tensors:
    the C library's choice, or ``grid`` where this module picks it."""
    dt = _DTYPE_CODE[dtype]
    grid = _grid_preferred(M, H, N, dt, torch.cuda.current_device())
    return _lib.query_schedule(M, H, N, dt, _lib.SCHED_GRID if grid else _lib.SCHED_AUTO)


def get_autotune_best_config(M: int, H: int) -> dict | None:
    """Describe the schedule chosen for a (M, H) seen before, else None (kernel.py:558-572).

    Keys ``BLOCK_M``, ``BLOCK_N``, ``BLOCK_K``, ``num_warps`` and ``num_stages`` carry
    the reference's meaning; ``schedule``, ``split_k``, ``grid`` and ``smem_bytes``
    describe the B200 kernel.
    """
    N = _seen_shapes.get((M, H))
    if N is None or not torch.cuda.is_available():
        return None
    info = schedule_info(M, H, N)
    return {
        "BLOCK_M": info["block_m"],
        "BLOCK_N": info["block_n"],
        "BLOCK_K": info["block_k"],
        "num_warps": info["threads"] // 32,
        "num_stages": info["stages"],
        "schedule": _lib.SCHEDULE_NAMES.get(info["schedule"], str(info["schedule"])),
        "split_k": info["split_k"],
        "grid": info["grid"],
        "smem_bytes": info["smem_bytes"],
        "uses_prepass": bool(info["uses_prepass"]),
    }


def device_status(device=None) -> int:
    """Synchronise the current stream and return/clear the library's device status bits."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        return _lib.device_status(torch.cuda.current_stream(dev).cuda_stream)
