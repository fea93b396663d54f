#!/usr/bin/env python
"""Benchmark of the fused residual add + RMSNorm + packed GQA QKV projection on B200.

One step = one fused op (one decoder layer's input RMSNorm + QKV projection) over one
batch of M tokens, on weight set ``i % sets``.  The default workload is the Llama-3-8B
layer shape at decode (H=4096, 32 q / 8 kv heads of 128 -> N_OUT=6144, bf16, M=16,
residual add with the updated residual returned).  32 distinct seeded weight sets
(1.61 GB) rotate so no weight is served from the 126 MB L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl ours`` (default) prints one JSON line with:
  value      whole-job HBM GB/s: algorithmic bytes of all ranks' steps / device time
             (max over ranks) of exactly K steps captured in one CUDA graph;
  e2e        the same metric through the public Python API with pinned host buffers:
             every step copies x and residual host->device, runs the op and copies the
             output and updated residual device->host, synchronising each step;
  roofline   achieved GB/s of the dominant kernel vs the measured HBM copy peak;
  cpu_baseline  the CPU oracle (a restatement of the reference's baseline.py) on a
             bounded sample of the same workload, rank 0 only at N=1;
  detail     the other configs measured the same way: Llama-3-8B decode M=1/4/16/64
             (bf16, fp16), Qwen2-7B decode M=1/16/64 (with and without residual),
             Llama-3-70B M=1/16/256, the post-attention gate/up shape (N=28672), prefill
             M=512/2048/8192 (TFLOPS), the unfused PyTorch path (cuBLAS) on the same
             inputs as the GPU comparator, an eager L2-flushed time of single Llama-3-8B
             decode steps (M=1/16) as a cross-check, a streaming-read bandwidth for context, and
             the FP8-weight path (e4m3 weight, Llama-3-8B decode M=1/16), and a
             4-layer Llama-3-8B stack (M=1/16) unpatched vs the integration patch's
             modes (Q/K/V, + MLP gate/up, cross-layer, + one-launch Q/K/V rotary split).
With N > 1 (torchrun) the layer is head-sharded column-parallel: each rank owns N/P
weight rows and computes them with replicated inputs; no collective runs inside the
timed region.  After timing, an NCCL all-gather reassembles one step for a check
against the unsharded result.

``--impl reference`` times the reference's CPU implementation (the oracle port of
baseline.py, all host threads) on the same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "fused-triton-rmsnorm-residual-qkv_b200"))

import torch  # noqa: E402

HBM_SPEC_GBS = 8000.0
BF16_SPEC_TFLOPS = 2250.0
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

WORKLOADS = {
    "llama3-8b-decode": dict(H=4096, n_q=32, n_kv=8, d=128, M=16, eps=1e-5, res=True, sets=32),
    "qwen2-7b-decode": dict(H=3584, n_q=28, n_kv=4, d=128, M=16, eps=1e-6, res=True, sets=32),
    "llama3-8b-prefill": dict(H=4096, n_q=32, n_kv=8, d=128, M=2048, eps=1e-5, res=True, sets=4),
    "llama3-70b": dict(H=8192, n_q=64, n_kv=8, d=128, M=1, eps=1e-5, res=True, sets=16),
    # post-attention residual add + RMSNorm + packed [W_gate; W_up] (N = 2 x 14336), as
    # 224 "heads" of 128 rows so the same set builder applies (single GPU only)
    "llama3-8b-mlp": dict(H=4096, n_q=224, n_kv=0, d=128, M=16, eps=1e-5, res=True, sets=8),
}


# ----------------------------------------------------------------------------- helpers
def algorithmic_bytes(M: int, H: int, N: int, res: bool, elem: int = 2) -> int:
    """Bytes a fused op must move at least: W, gain, x, residual, output, updated residual."""
    return elem * (N * H + H + M * H + (M * H if res else 0) + M * N + (M * H if res else 0))


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS, "source": "fallback"}


def profile_traffic(name: str):
    """DRAM bytes per launch recorded from an ncu capture in profiles/<name>.md, if any."""
    p = ROOT / "profiles" / f"{name}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", p.read_text())
    return int(m.group(1)) if m else None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.001):
        self.ok = False
        self.samples: list[tuple[int, int]] = []
        self.period = period_s
        try:
            import pynvml

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device_index)
            handle = None
            uuid = str(getattr(props, "uuid", ""))
            if uuid:
                uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
                try:
                    handle = pynvml.nvmlDeviceGetHandleByUUID(uuid)
                except Exception:
                    handle = None
            if handle is None:
                handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.nvml, self.h = pynvml, handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report why
            self.err = str(e)
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                clk = self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM)
                rsn = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((clk, rsn))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "err", "")}
        loaded = [s for s in self.samples if not (s[1] & 0x1)] or self.samples
        reasons = set()
        for _, r in loaded:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median([c for c, _ in loaded]) if loaded else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons), "samples": len(loaded)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ----------------------------------------------------------------------------- inputs
def make_sets(wl: dict, M: int, dtype, dev, world: int, rank: int, sets: int):
    """Per-set seeded inputs on the device: (x, residual, gain, local weight)."""
    from triton_fused_rmsnorm_qkv.sharding import HeadLayout, shard_qkv_weight

    layout = HeadLayout(wl["n_q"], wl["n_kv"], wl["d"])
    H, N = wl["H"], layout.n_out
    out = []
    for i in range(sets):
        g = torch.Generator(device=dev).manual_seed(1000 + i)
        x = torch.randn(1, M, H, generator=g, device=dev, dtype=torch.float32).to(dtype)
        r = torch.randn(1, M, H, generator=g, device=dev, dtype=torch.float32).to(dtype) if wl["res"] else None
        gain = (1.0 + 0.1 * torch.randn(H, generator=g, device=dev, dtype=torch.float32)).to(dtype)
        w = (0.02 * torch.randn(N, H, generator=g, device=dev, dtype=torch.float32)).to(dtype)
        if world > 1:
            w = shard_qkv_weight(w, layout, rank, world)
        out.append((x, r, gain, w))
    return out, layout


def time_graph(fn_step, steps: int, warmup: int, dev, sampler: ClockSampler | None = None, barrier=None,
               replays: int = 1, min_seconds: float = 0.0, stats: dict | None = None):
    """Warm up, capture `steps` calls of fn_step(i) in one CUDA graph, and time replays of it.

    Each replay is timed with its own CUDA events on the capture stream; the result is the
    median over the replays, in milliseconds for the K steps.  At least `replays` replays
    run, and more if needed to keep the GPU busy for `min_seconds` (so that a clock sampler
    sees the load).  With `barrier`, the ranks meet before the first and after the last
    replay.  `stats` (if given) receives the replay count and the first replay's time."""
    for i in range(warmup):
        fn_step(i)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fn_step(0)  # allocator warm-up on the capture stream
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                fn_step(i)
    torch.cuda.synchronize(dev)
    graph.replay()  # first replay uploads the graph
    torch.cuda.synchronize(dev)
    if min_seconds > 0:  # size the replay count from one timed replay
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        replays = max(replays, int(math.ceil(min_seconds * 1e3 / max(e0.elapsed_time(e1), 1e-3))))
    if barrier is not None:  # every rank runs the same number of replays
        t = torch.tensor([replays], device=dev)
        barrier(t)
        replays = int(t.item())
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(replays)]
    if barrier:
        barrier()
    torch.cuda.synchronize(dev)
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        with torch.cuda.stream(stream):
            for e0, e1 in evs:
                e0.record(stream)
                graph.replay()
                e1.record(stream)
        torch.cuda.synchronize(dev)
    if barrier:
        barrier()
    times = [e0.elapsed_time(e1) for e0, e1 in evs]
    if stats is not None:
        stats.update(replays=replays, first_replay_ms=times[0], min_replay_ms=min(times), max_replay_ms=max(times))
    del graph
    return statistics.median(times)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def op_step_fn(sets, eps, M, schedule=None):
    from triton_fused_rmsnorm_qkv import fused_add_rmsnorm_matmul

    S = len(sets)

    def step(i):
        x, r, g, w = sets[i % S]
        fused_add_rmsnorm_matmul(x, r, g, w, eps, schedule=schedule, static_weights=True)

    return step


# ----------------------------------------------------------------------------- CPU legs
def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo), or the platform's description."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or platform.machine()


def cpu_time_op(wl: dict, M: int, dtype, seconds: float, threads: int):
    """Median seconds per op of the CPU oracle on one seeded set of the workload, and the
    number of ops timed: ``torch.utils.benchmark.Timer.blocked_autorange`` over about
    ``seconds`` with ``threads`` threads."""
    from torch.utils import benchmark

    sys.path.insert(0, str(ROOT))
    from oracle import forward, make_case

    N = wl["n_q"] * wl["d"] + 2 * wl["n_kv"] * wl["d"]
    x, r, g, w = make_case(M, wl["H"], N, dtype, 1000, wl["res"])
    timer = benchmark.Timer(stmt="forward(x, r, g, w, eps)", num_threads=threads,
                            globals=dict(forward=forward, x=x, r=r, g=g, w=w, eps=wl["eps"]))
    m = timer.blocked_autorange(min_run_time=seconds)
    return m.median, len(m.times) * m.number_per_run


def run_reference(args, wl: dict, M: int) -> dict:
    """--impl reference: the oracle port of baseline.py on all host threads."""
    dtype = torch.bfloat16
    N = wl["n_q"] * wl["d"] + 2 * wl["n_kv"] * wl["d"]
    bytes_step = algorithmic_bytes(M, wl["H"], N, wl["res"])
    threads = os.cpu_count() or 1
    sys.path.insert(0, str(ROOT))
    from oracle import forward, make_case

    torch.set_num_threads(threads)
    x, r, g, w = make_case(M, wl["H"], N, dtype, 1000, wl["res"])
    for _ in range(args.warmup):
        forward(x, r, g, w, wl["eps"])
    t0 = time.perf_counter()
    for _ in range(args.steps):
        forward(x, r, g, w, wl["eps"])
    dt = time.perf_counter() - t0
    gbs = bytes_step * args.steps / dt / 1e9
    sample = f"{args.steps} full ops of the workload (M={M}, H={wl['H']}, N={N}, bf16) on the CPU"
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 6),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)",
        "config": {"workload": f"{args.workload} M={M}", "H": wl["H"], "N_OUT": N, "M": M,
                   "has_residual": wl["res"]},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


METRIC = "fused-op µs & HBM GB/s (% of 8 TB/s) at M=1/16, Llama-3-8B shape; prefill TFLOPS"


# ----------------------------------------------------------------------------- detail
# (label, workload, M, dtype name, has residual, weight sets, comparator).  The MLP entry
# is the same op on the post-attention side of a Llama-3-8B layer: residual add +
# post_attention_layernorm + the packed [W_gate; W_up] projection (N = 2 x 14336).
DETAIL = [
    ("llama3-8b_decode_M1", "llama3-8b-decode", 1, "bf16", True, 32, True),
    ("llama3-8b_decode_M4", "llama3-8b-decode", 4, "bf16", True, 32, False),
    ("llama3-8b_decode_M16", "llama3-8b-decode", 16, "bf16", True, 32, True),
    ("llama3-8b_decode_M64", "llama3-8b-decode", 64, "bf16", True, 32, False),
    ("llama3-8b_decode_M1_fp16", "llama3-8b-decode", 1, "fp16", True, 32, False),
    ("llama3-8b_decode_M16_fp16", "llama3-8b-decode", 16, "fp16", True, 32, False),
    ("qwen2-7b_decode_M1", "qwen2-7b-decode", 1, "bf16", True, 32, False),
    ("qwen2-7b_decode_M16", "qwen2-7b-decode", 16, "bf16", True, 32, False),
    ("qwen2-7b_decode_M64", "qwen2-7b-decode", 64, "bf16", True, 32, False),
    ("qwen2-7b_decode_M16_no_residual", "qwen2-7b-decode", 16, "bf16", False, 32, False),
    ("llama3-70b_M1", "llama3-70b", 1, "bf16", True, 16, False),
    ("llama3-70b_M16", "llama3-70b", 16, "bf16", True, 16, False),
    ("llama3-70b_M256", "llama3-70b", 256, "bf16", True, 8, False),
    ("llama3-8b_mlp_gate_up_M1", "llama3-8b-mlp", 1, "bf16", True, 8, False),
    ("llama3-8b_mlp_gate_up_M16", "llama3-8b-mlp", 16, "bf16", True, 8, False),
    ("llama3-8b_prefill_M512", "llama3-8b-prefill", 512, "bf16", True, 4, False),
    ("llama3-8b_prefill_M2048", "llama3-8b-prefill", 2048, "bf16", True, 4, True),
    ("llama3-8b_prefill_M8192", "llama3-8b-prefill", 8192, "bf16", True, 4, False),
]


def torch_step_fn(sets, eps):
    """The unfused PyTorch path (the reference's baseline.py semantics) on the GPU."""
    from triton_fused_rmsnorm_qkv import rmsnorm_residual_qkv

    S = len(sets)

    def step(i):
        x, r, g, w = sets[i % S]
        rmsnorm_residual_qkv(x, r, g, w, eps)

    return step


def load_reference_triton():
    """The reference's own package (its Triton kernels), installed unmodified under
    baseline/_ref, imported under a private module name so that it cannot shadow this
    repository's package of the same name.  None when it or Triton is not present."""
    import importlib.util

    pkg = ROOT / "baseline" / "_ref" / "triton_fused_rmsnorm_qkv"
    if not (pkg / "__init__.py").exists():
        return None
    try:
        import triton  # noqa: F401
    except ImportError:
        return None
    name = "_reference_triton_fused_rmsnorm_qkv"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def run_reference_triton_detail(dev, peaks: dict, autotune: bool) -> dict:
    """The reference's Triton kernels on this GPU, as a comparator outside the product path:
    ``fused_rmsnorm_residual_matmul`` (autotuned on its first call per shape, during the
    warm-up) or its ``_fixed`` variant, at Llama-3-8B M = 1 / 16 / 2048, graph-timed like the
    other rows.  The reference returns no updated residual, so its bytes omit that write."""
    ref = load_reference_triton()
    if ref is None:
        return {"unavailable": "the reference package (baseline/_ref) or Triton is not installed here"}
    fn = ref.fused_rmsnorm_residual_matmul if autotune else ref.fused_rmsnorm_residual_matmul_fixed
    out = {"entry_point": fn.__name__, "source": "baseline/_ref (the reference, installed unmodified)"}
    for mm, n_sets in ((1, 32), (16, 32), (2048, 4)):
        wl = dict(WORKLOADS["llama3-8b-decode"], sets=n_sets)
        ss, layout = make_sets(wl, mm, torch.bfloat16, dev, 1, 0, n_sets)
        H, N = wl["H"], layout.n_out

        def step(i, ss=ss):
            x, r, g, w = ss[i % len(ss)]
            fn(x, r, g, w, wl["eps"])

        k = 200 if mm <= 64 else 40
        t0 = time.perf_counter()
        try:
            t_ms = time_graph(step, k, 3, dev) / k
        except Exception as e:  # a Triton compile or launch problem on this part
            out[f"M{mm}"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
            continue
        b = algorithmic_bytes(mm, H, N, True) - 2 * mm * H  # no updated residual written
        out[f"M{mm}"] = {"us": round(t_ms * 1e3, 3), "GB/s": round(b / t_ms / 1e6, 1),
                         "pct_of_measured_hbm": round(100 * b / t_ms / 1e6 / peaks["hbm_gbs"], 2),
                         "TFLOPS": round(2.0 * mm * N * H / t_ms / 1e9, 1),
                         "setup_and_timing_s": round(time.perf_counter() - t0, 1)}
        del ss
    return out


def hbm_read_peak_gbs(dev) -> float:
    """Streaming read bandwidth of a 4 GiB bf16 tensor (torch.sum), for context beside the
    measured copy peak: a decode op is almost entirely a read."""
    t = torch.ones(2 << 30, dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        t.sum()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record()
    for _ in range(10):
        t.sum()
    e1.record()
    torch.cuda.synchronize(dev)
    gbs = t.numel() * 2 * 10 / (e0.elapsed_time(e1) / 1e3) / 1e9
    del t
    return gbs


def eager_flushed_us(fn_step, n: int, dev) -> float:
    """Median microseconds of one eager step timed alone with CUDA events, L2 flushed before
    each: a 256 MB memset (twice the L2) runs first, which also keeps the GPU queue ahead
    of the host, so the events bracket the step's kernels and not the host's launch cost.
    A cross-check of the graph-timed numbers: no overlap with a preceding kernel, cold L2."""
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for i in range(n + 3):
        flush.zero_()
        e0.record()
        fn_step(i)
        e1.record()
        torch.cuda.synchronize(dev)
        if i >= 3:
            times.append(e0.elapsed_time(e1) * 1e3)
    del flush
    return statistics.median(times)


def after_other_kernel_us(fn_step, steps: int, dev) -> float:
    """Microseconds one step adds to a CUDA graph when it follows an ordinary PyTorch kernel
    (an elementwise op on a 4 KB tensor, launched without programmatic dependent launch), as in
    a model whose preceding op is not this library's: graph of [other, step] x K minus graph of
    [other] x K.  Nothing of the step overlaps a preceding step; the launch itself is pipelined
    by the graph, as in a graph-captured model."""
    other = torch.zeros(1024, device=dev)

    def pair(i):
        other.mul_(1.0)
        fn_step(i)

    t_pair = time_graph(pair, steps, 5, dev, replays=20) / steps
    t_other = time_graph(lambda i: other.mul_(1.0), steps, 5, dev, replays=20) / steps
    return (t_pair - t_other) * 1e3


def eager_event_floor_us(dev, n: int = 50) -> float:
    """What the eager, event-bracketed measurement of eager_flushed_us reports for a kernel that
    does almost nothing (the same 4 KB elementwise op), after the same 256 MB memset: the launch
    and event overhead contained in every eager_flushed_us figure."""
    other = torch.zeros(1024, device=dev)
    return eager_flushed_us(lambda i: other.mul_(1.0), n, dev)


def run_detail(wl_default: dict, dev, peaks: dict, args_triton_comparator: str = "autotune") -> dict:
    from triton_fused_rmsnorm_qkv import _lib
    from triton_fused_rmsnorm_qkv.kernel import schedule_info

    dtypes = {"bf16": (torch.bfloat16, _lib.BF16), "fp16": (torch.float16, _lib.F16)}
    detail = {"hbm_read_peak_gbs_torch_sum": round(hbm_read_peak_gbs(dev), 1)}
    for label, wname, mm, dname, res, n_sets, comparator in DETAIL:
        wl = dict(WORKLOADS[wname], res=res, sets=n_sets)
        dt, _ = dtypes[dname]
        ss, layout = make_sets(wl, mm, dt, dev, 1, 0, n_sets)
        H, N = wl["H"], layout.n_out
        k = 2000 if mm <= 64 else (200 if mm <= 512 else (40 if mm <= 2048 else 12))
        t_ms = time_graph(op_step_fn(ss, wl["eps"], mm), k, 5, dev) / k
        b = algorithmic_bytes(mm, H, N, res)
        fl = 2.0 * mm * N * H
        entry = {"M": mm, "H": H, "N": N, "dtype": dname, "residual": res, "us": round(t_ms * 1e3, 3),
                 "GB/s": round(b / t_ms / 1e6, 1), "pct_of_measured_hbm": round(100 * b / t_ms / 1e6 / peaks["hbm_gbs"], 2),
                 "TFLOPS": round(fl / t_ms / 1e9, 1),
                 "pct_of_measured_bf16": round(100 * fl / t_ms / 1e9 / peaks["bf16_tflops"], 2),
                 "schedule": _lib.SCHEDULE_NAMES[schedule_info(mm, H, N, dt)["schedule"]]}
        if comparator:
            t_ref = time_graph(torch_step_fn(ss, wl["eps"]), k, 5, dev) / k
            entry["torch_unfused_us"] = round(t_ref * 1e3, 3)
            entry["speedup_vs_torch_unfused"] = round(t_ref / t_ms, 2)
            if mm <= 64:
                entry["eager_l2_flushed_us"] = round(eager_flushed_us(op_step_fn(ss, wl["eps"], mm), 50, dev), 3)
                entry["eager_event_floor_us"] = round(eager_event_floor_us(dev), 3)
                entry["graph_after_other_kernel_us"] = round(after_other_kernel_us(op_step_fn(ss, wl["eps"], mm),
                                                                                   200, dev), 3)
        detail[label] = entry
        del ss
    detail.update(run_fp8w_detail(dev, peaks))
    detail["llama3-8b_decode_rope"] = run_rope_detail(dev)
    if args_triton_comparator != "off":
        detail["reference_triton"] = run_reference_triton_detail(dev, peaks, args_triton_comparator == "autotune")
    detail["llama3-8b_layer_stack"] = run_layer_stack(dev)
    detail["llama3-8b_kv_cache_decode"] = run_kv_decode(dev)
    return detail


def run_fp8w_detail(dev, peaks: dict) -> dict:
    """The FP8-weight path (e4m3 weight + fp32 row scale, quantize_weight_e4m3) on the
    Llama-3-8B decode shape, graph-timed like the rows above.  Bytes: the one-byte weight
    and its scales plus the 16-bit activations, gain, output and updated residual."""
    from triton_fused_rmsnorm_qkv import fused_add_rmsnorm_matmul_fp8w, quantize_weight_e4m3

    out = {}
    wl = dict(WORKLOADS["llama3-8b-decode"], sets=32)
    for mm in (1, 16):
        ss, layout = make_sets(wl, mm, torch.bfloat16, dev, 1, 0, wl["sets"])
        q8 = [(x, r, g, *quantize_weight_e4m3(w)) for (x, r, g, w) in ss]
        del ss

        def step(i):
            x, r, g, w8, sc = q8[i % len(q8)]
            fused_add_rmsnorm_matmul_fp8w(x, r, g, w8, sc, wl["eps"], static_weights=True)

        t_ms = time_graph(step, 2000, 5, dev) / 2000
        H, N = wl["H"], layout.n_out
        b = N * H + 4 * N + algorithmic_bytes(mm, H, 0, True) + 2 * mm * N  # + the output
        out[f"llama3-8b_decode_fp8w_M{mm}"] = {
            "M": mm, "H": H, "N": N, "dtype": "bf16 activations, e4m3 weight", "us": round(t_ms * 1e3, 3),
            "GB/s": round(b / t_ms / 1e6, 1), "pct_of_measured_hbm": round(100 * b / t_ms / 1e6 / peaks["hbm_gbs"], 2)}
        del q8
        torch.cuda.empty_cache()
    return out


def run_rope_detail(dev, ms=(1, 16)) -> dict:
    """The Q/K/V split + rotary embedding (llama3_patch.py:148-168) on the Llama-3-8B decode
    shape, M sequences of one token each at their own positions, graph-timed like the rows
    above: the projection alone, the projection followed by the separate rotary split
    (two launches), and the rotary split in the projection's epilogue (one launch)."""
    from triton_fused_rmsnorm_qkv import fused_add_rmsnorm_matmul, fused_add_rmsnorm_qkv_rope, qkv_rope_split

    wl = dict(WORKLOADS["llama3-8b-decode"], sets=32)
    out = {"unit": "us per step", "shape": "M sequences x 1 token, H 4096, 32 q / 8 kv heads of 128, bf16"}
    for mm in ms:
        ss, layout = make_sets(wl, mm, torch.bfloat16, dev, 1, 0, wl["sets"])
        gen = torch.Generator(device=dev).manual_seed(5)
        pos = torch.randint(0, 4096, (mm,), generator=gen, device=dev).float()
        inv = 1.0 / (500000.0 ** (torch.arange(0, wl["d"], 2, device=dev).float() / wl["d"]))
        ang = torch.cat([pos[:, None] * inv[None]] * 2, dim=-1)[:, None, :]  # (M, 1, d)
        cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
        sets = [(x.view(mm, 1, -1), r.view(mm, 1, -1), g, w) for (x, r, g, w) in ss]
        del ss
        nq, nkv, eps = wl["n_q"], wl["n_kv"], wl["eps"]

        def alone(i):
            x, r, g, w = sets[i % len(sets)]
            fused_add_rmsnorm_matmul(x, r, g, w, eps, static_weights=True)

        def two(i):
            x, r, g, w = sets[i % len(sets)]
            qkv, _ = fused_add_rmsnorm_matmul(x, r, g, w, eps, static_weights=True)
            qkv_rope_split(qkv, cos, sin, nq, nkv)

        def one(i):
            x, r, g, w = sets[i % len(sets)]
            fused_add_rmsnorm_qkv_rope(x, r, g, w, cos, sin, nq, nkv, eps=eps, static_weights=True)

        row = {}
        for name, fn in (("projection_only", alone), ("projection_then_rope_split", two), ("fused_rope", one)):
            row[name] = round(time_graph(fn, 1000, 5, dev, replays=10) / 1000 * 1e3, 3)
        row["fused_rope_over_projection_only"] = round(row["fused_rope"] - row["projection_only"], 3)
        out[f"M{mm}"] = row
        del sets
        torch.cuda.empty_cache()
    return out


def run_layer_stack(dev, n_layers: int = 4, ms=(1, 16), steps: int = 50) -> dict:
    """Model-level check of the integration: a stack of Llama-3-8B decoder layers (random
    init, bf16, no KV cache, causal attention over the M tokens) and the final norm,
    graph-timed per forward of M tokens.  Unpatched PyTorch against the patch in its three
    modes: Q/K/V only (the reference's patch), + post-attention add/norm/gate-up,
    cross-layer (each layer's MLP residual add fused into the next layer's input call), and
    cross-layer with the Q/K/V split + rotary embedding in one launch."""
    from contextlib import nullcontext

    from integration import build_llama3_8b, fused_patch

    model = build_llama3_8b(dtype=torch.bfloat16, device=str(dev), num_hidden_layers=n_layers)
    inner = model.model
    modes = (("unpatched", None), ("qkv", {}), ("qkv+mlp", {"mlp": True}), ("cross-layer", {"cross_layer": True}),
             ("cross-layer+rope", {"cross_layer": True, "rope": True}))
    out = {"layers": n_layers, "steps": steps, "unit": "us per forward of M tokens through all layers"}
    with torch.no_grad():
        for M in ms:
            gen = torch.Generator(device=dev).manual_seed(5)
            h0 = torch.randn(1, M, WORKLOADS["llama3-8b-decode"]["H"], generator=gen, device=dev, dtype=torch.bfloat16)
            pos = torch.arange(M, device=dev)[None]
            pe = inner.rotary_emb(h0, pos)

            def step(i):
                x = h0
                for layer in inner.layers:
                    x = layer(x, attention_mask=None, position_ids=pos, position_embeddings=pe)
                return inner.norm(x)

            row = {}
            for name, kw in modes:
                with (nullcontext() if kw is None else fused_patch(model, **kw)):
                    row[name] = round(time_graph(step, steps, 3, dev) / steps * 1e3, 2)
            out[f"M{M}"] = row
    del model, inner
    torch.cuda.empty_cache()
    return out


def run_kv_decode(dev, n_layers: int = 4, batches=(1, 16), prompt_len: int = 128, n_new: int = 256,
                  repeats: int = 3) -> dict:
    """Greedy decode with a static KV cache on a Llama-3-8B-shaped model (random init, bf16,
    ``n_layers`` decoder layers, full vocabulary): the methodology of the reference's
    e2e_decode.py (prompt 128, 256 new tokens, batch 1 and 16, tokens per second over the
    decode phase) with each decode step replayed from a CUDA graph
    (integration.GraphedGreedyDecoder).  Unpatched against the patch's modes; each patched
    run's tokens are compared with the unpatched run's.  A random-init model's next-token
    distribution is nearly flat, so a last-bit difference in one step can flip a greedy
    choice and the two free-running sequences part for good; each mode is therefore also
    run teacher-forced on the unpatched tokens, and the rows report how often its greedy
    choice agrees with the unpatched one given the same prefix, and the largest logit
    difference."""
    from contextlib import nullcontext

    from integration import GraphedGreedyDecoder, build_llama3_8b, fused_patch

    model = build_llama3_8b(dtype=torch.bfloat16, device=str(dev), num_hidden_layers=n_layers)
    modes = (("unpatched", None), ("qkv", {}), ("cross-layer+rope", {"cross_layer": True, "rope": True}))
    out = {"layers": n_layers, "prompt_len": prompt_len, "new_tokens": n_new,
           "unit": "decode tokens per second (batch x steps / CUDA-event time of the graph replays)"}
    with torch.no_grad():
        for B in batches:
            gen = torch.Generator(device=dev).manual_seed(11)
            prompt = torch.randint(0, model.config.vocab_size, (B, prompt_len), generator=gen, device=dev)
            row, ref_tokens, ref_forced = {}, None, None
            for name, kw in modes:
                with (nullcontext() if kw is None else fused_patch(model, **kw)):
                    dec = GraphedGreedyDecoder(model, B, prompt_len + n_new)
                    secs = []
                    for _ in range(repeats):
                        tokens = dec.generate(prompt, n_new)
                        secs.append(dec.decode_seconds)
                    forced = dec.forced_logits(prompt, tokens if ref_tokens is None else ref_tokens)
                steps = n_new - 2
                t = statistics.median(secs)
                entry = {"tok_per_s": round(B * steps / t, 1), "us_per_step": round(t / steps * 1e6, 2)}
                if ref_tokens is None:
                    ref_tokens, ref_forced = tokens, forced
                    entry["teacher_forced_argmax_equals_own_tokens"] = round(
                        float((forced.argmax(-1) == tokens).float().mean()), 4)
                else:
                    same = (tokens == ref_tokens).all(dim=0)
                    entry["tokens_equal_unpatched"] = bool(same.all())
                    entry["steps_equal_before_first_difference"] = int(same.long().cumprod(0).sum())
                    entry["teacher_forced_argmax_agreement"] = round(
                        float((forced.argmax(-1) == ref_tokens).float().mean()), 4)
                    entry["teacher_forced_max_abs_logit_diff"] = round(float((forced - ref_forced).abs().max()), 4)
                    entry["logit_std"] = round(float(ref_forced.std()), 4)
                del forced
                row[name] = entry
            out[f"batch{B}"] = row
            del ref_forced
    del model
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- GPU arm
# Llama-3-70B rows of the head-sharded run (N > 1): (label, M, weight sets).
SHARDED_DETAIL = [("llama3-70b_M1", 1, 16), ("llama3-70b_M16", 16, 16), ("llama3-70b_M256", 256, 8)]


def reference_unsharded(wl: dict, M: int, dtype, dev):
    """Set 0 of make_sets with the whole (unsharded) weight, rebuilt from the same seed."""
    gen = torch.Generator(device=dev).manual_seed(1000)
    torch.randn(1, M, wl["H"], generator=gen, device=dev)
    if wl["res"]:
        torch.randn(1, M, wl["H"], generator=gen, device=dev)
    torch.randn(wl["H"], generator=gen, device=dev)
    N = wl["n_q"] * wl["d"] + 2 * wl["n_kv"] * wl["d"]
    return (0.02 * torch.randn(N, wl["H"], generator=gen, device=dev)).to(dtype)


def shard_check(pg, sets, layout, wl: dict, M: int, dtype, dev, rank: int, world: int):
    """Untimed check of a head-sharded step: every rank computes set 0 of its shard, an NCCL
    all-gather reassembles Q/K/V, and rank 0 compares it with the unsharded op.  The updated
    residual (computed by every rank from replicated inputs) must be bit-identical."""
    from triton_fused_rmsnorm_qkv import fused_add_rmsnorm_matmul, fused_rmsnorm_residual_matmul
    from triton_fused_rmsnorm_qkv.sharding import gather_qkv

    x, r, g, w_loc = sets[0]
    out_loc, hid_loc = fused_add_rmsnorm_matmul(x, r, g, w_loc, wl["eps"])
    full = gather_qkv(out_loc, layout)
    hids = [torch.empty_like(hid_loc) for _ in range(world)]
    pg.all_gather(hids, hid_loc.contiguous())
    result = None
    if rank == 0:
        ref = fused_rmsnorm_residual_matmul(x, r, g, reference_unsharded(wl, M, dtype, dev), wl["eps"])
        d = full.float() - ref.float()
        result = {"max_abs_vs_unsharded": float(d.abs().max()),
                  "rel_l2_vs_unsharded": float(d.norm() / ref.float().norm()),
                  "residual_bit_identical_across_ranks":
                      all(torch.equal(h.view(torch.int16), hids[0].view(torch.int16)) for h in hids),
                  "gathered_with": "nccl all_gather"}
    pg.barrier()
    return result


def run_sharded_detail(pg, barrier, dev, rank: int, world: int, peaks: dict) -> dict:
    """Llama-3-70B layer head-sharded over the ranks at M = 1 / 16 / 256: graph-timed like the
    headline (max over ranks), aggregate and per-GPU throughput, and a shard check each."""
    from triton_fused_rmsnorm_qkv import _lib
    from triton_fused_rmsnorm_qkv.kernel import schedule_info

    out = {}
    for label, mm, n_sets in SHARDED_DETAIL:
        wl = dict(WORKLOADS["llama3-70b"], sets=n_sets)
        ss, layout = make_sets(wl, mm, torch.bfloat16, dev, world, rank, n_sets)
        H, N_glob, N_loc = wl["H"], layout.n_out, ss[0][3].shape[0]
        k = 200 if mm <= 64 else 50
        t = torch.tensor([time_graph(op_step_fn(ss, wl["eps"], mm), k, 5, dev, barrier=barrier, replays=20) / k],
                         device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        t_ms = float(t.item())
        b_rank = algorithmic_bytes(mm, H, N_loc, True)
        fl_rank = 2.0 * mm * N_loc * H
        entry = {"M": mm, "H": H, "N": N_glob, "N_per_gpu": N_loc, "us": round(t_ms * 1e3, 3),
                 "GB/s_aggregate": round(world * b_rank / t_ms / 1e6, 1), "GB/s_per_gpu": round(b_rank / t_ms / 1e6, 1),
                 "pct_of_measured_hbm_per_gpu": round(100 * b_rank / t_ms / 1e6 / peaks["hbm_gbs"], 2),
                 "TFLOPS_aggregate": round(world * fl_rank / t_ms / 1e9, 1),
                 "TFLOPS_per_gpu": round(fl_rank / t_ms / 1e9, 1),
                 "pct_of_measured_bf16_per_gpu": round(100 * fl_rank / t_ms / 1e9 / peaks["bf16_tflops"], 2),
                 "schedule": _lib.SCHEDULE_NAMES[schedule_info(mm, H, N_loc)["schedule"]]}
        chk = shard_check(pg, ss, layout, wl, mm, torch.bfloat16, dev, rank, world)
        if chk is not None:
            entry["shard_check"] = chk
        out[label] = entry
        del ss
        torch.cuda.empty_cache()
    return out


def run_e2e(sets, wl: dict, M: int, H: int, N_loc: int, dtype, dev, args, pg) -> dict:
    """The metric through the public API on every rank: each step copies that step's x and
    residual from pinned host memory to the device, runs the op on the rank's shard and
    copies its output and updated residual back, synchronising every step.  Time per step
    is the max over ranks of the CUDA-event (or, if longer, wall-clock) time."""
    from triton_fused_rmsnorm_qkv import fused_add_rmsnorm_matmul

    x0, r0, g0, w0 = sets[0]
    # A step's inputs (x, then the residual) sit in one pinned host buffer and go over in
    # one copy; its results (the output, then the updated residual) are written by the call
    # into one device buffer (out= / residual_out=) and come back in one copy.  Each DMA
    # copy costs several microseconds of latency whatever its size.
    n_in = 2 if r0 is not None else 1
    in_h = torch.empty(n_in, M, H, dtype=dtype).pin_memory()
    in_h[0].copy_(x0[0].cpu())
    if r0 is not None:
        in_h[1].copy_(r0[0].cpu())
    res_h = torch.empty(M * N_loc + M * H, dtype=dtype).pin_memory()
    in_d = torch.empty(n_in, M, H, dtype=dtype, device=dev)
    res_d = torch.empty(M * N_loc + M * H, dtype=dtype, device=dev)
    xd = in_d[0:1]
    rd = in_d[1:2] if r0 is not None else None
    out_d, hid_d = res_d[:M * N_loc].view(1, M, N_loc), res_d[M * N_loc:].view(1, M, H)
    e2e_steps = max(10, min(args.steps, 2000))

    def e2e_step(i):
        _, _, g_i, w_i = sets[i % len(sets)]
        in_d.copy_(in_h, non_blocking=True)
        fused_add_rmsnorm_matmul(xd, rd, g_i, w_i, wl["eps"], static_weights=True, out=out_d, residual_out=hid_d)
        res_h.copy_(res_d, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()

    for i in range(max(3, args.warmup)):
        e2e_step(i)
    if pg is not None:
        pg.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    ev0.record()
    w0t = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i)
    ev1.record()
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - w0t
    t = torch.tensor([max(ev0.elapsed_time(ev1), wall * 1e3) / e2e_steps], device=dev)
    world = 1
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        world = pg.get_world_size()
    e2e_ms = float(t.item())
    h2d = in_h.numel() * 2
    d2h = res_h.numel() * 2
    job_bytes = algorithmic_bytes(M, H, N_loc, wl["res"]) * world
    return {"value": round(job_bytes / (e2e_ms / 1e3) / 1e9, 3), "unit": "GB/s",
            "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
            "h2d_bytes_per_step_per_gpu": h2d, "d2h_bytes_per_step_per_gpu": d2h,
            "ms_per_step": round(e2e_ms, 6), "steps": e2e_steps,
            "path": "fused_add_rmsnorm_matmul (public API) on every rank: x and residual in from one pinned "
                    "host buffer (one copy), the rank's output and updated residual written by the call into one "
                    "device buffer (out= / residual_out=) and read back in one copy, synchronised every step; "
                    "job bytes over the max-over-ranks time",
            "n_gpus_used": world}


def run_ours(args, wl: dict, M: int) -> dict | None:
    world, rank, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # Rank 0 prints exactly one JSON line on stdout.  NCCL's own messages go to stderr
        # unless the caller chose a destination, and its version banner, which it writes to
        # the process's standard output when the communicator comes up, is kept off stdout
        # by pointing file descriptor 1 at stderr until the first collective has run.
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
            dist.barrier()
            torch.cuda.synchronize(dev)
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)
        pg = dist

    def barrier(t=None):
        """Meet the other ranks; with a tensor, also take its max over the ranks."""
        if pg is None:
            return
        if t is not None:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        else:
            pg.barrier()

    dtype = torch.bfloat16
    sets, layout = make_sets(wl, M, dtype, dev, world, rank, wl["sets"])
    H, N_glob = wl["H"], layout.n_out
    N_loc = sets[0][3].shape[0]
    peaks = measured_peaks()

    # ---- main timed region: the K-step graph replayed (at least 50 times, and for at least
    # 0.3 s so the clock sampler sees the load); median replay, max over ranks
    sampler = ClockSampler(local)
    step = op_step_fn(sets, wl["eps"], M)
    tstats: dict = {}
    ms = time_graph(step, args.steps, args.warmup, dev, sampler=sampler, barrier=barrier, replays=50,
                    min_seconds=0.3, stats=tstats)
    t = torch.tensor([ms], device=dev)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms_max = float(t.item())
    # algorithmic bytes of all ranks (each reads the replicated x / residual / gain and
    # writes the replicated updated residual; the weight and output are split)
    per_rank = algorithmic_bytes(M, H, N_loc, wl["res"])
    job_bytes = per_rank * world
    step_s = ms_max / 1e3 / args.steps
    value = job_bytes / step_s / 1e9
    from triton_fused_rmsnorm_qkv import _lib

    from triton_fused_rmsnorm_qkv.kernel import schedule_info

    sched = schedule_info(M, H, N_loc)
    launches = tstats["replays"] * args.steps * (2 if sched["uses_prepass"] else 1)

    # ---- verification of the sharded run (untimed): NCCL all-gather vs unsharded op
    check = shard_check(pg, sets, layout, wl, M, dtype, dev, rank, world) if world > 1 else None

    # ---- e2e through the public API with pinned host buffers, on every rank
    e2e = run_e2e(sets, wl, M, H, N_loc, dtype, dev, args, pg)

    # ---- Llama-3-70B head-sharded rows (N > 1)
    sharded = run_sharded_detail(pg, barrier, dev, rank, world, peaks) if world > 1 and not args.no_detail else {}

    if rank != 0:
        if pg is not None:
            pg.destroy_process_group()
        return None

    # ---- detail: the metric's other points and the other configs, timed the same way,
    # with the unfused PyTorch path (cuBLAS) as the GPU comparator (N=1 only)
    detail = {}
    if world == 1 and not args.no_detail:
        detail = run_detail(wl, dev, peaks, args.triton_comparator)
        torch.cuda.empty_cache()
    detail.update(sharded)

    # ---- CPU baseline (rank 0, N=1): the oracle on a bounded sample, all host threads and one
    cpu = None
    if world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        sec, n = cpu_time_op(wl, M, dtype, args.cpu_seconds, threads)
        sec1, n1 = cpu_time_op(wl, M, dtype, max(2.0, args.cpu_seconds / 3), 1)
        b_glob = algorithmic_bytes(M, H, N_glob, wl["res"])
        cpu = {"value": round(b_glob / sec / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "one_thread_value": round(b_glob / sec1 / 1e9, 3), "cpu_model": cpu_model(),
               "torch_threads": threads,
               "method": "torch.utils.benchmark.Timer.blocked_autorange, median",
               "sample": f"{n} ops of the same workload (M={M}, H={H}, N={N_glob}, bf16, one seeded set) over "
                         f"~{args.cpu_seconds:.0f} s on {threads} threads, median op {sec * 1e3:.3f} ms; "
                         f"{n1} ops on 1 thread, median op {sec1 * 1e3:.3f} ms"}

    # ncu DRAM bytes of the dominant kernel, captured at N = 1 on the whole weight; at N > 1
    # a rank reads 1/N of the weight, so the capture is scaled by this rank's algorithmic bytes.
    def traffic(name: str):
        t1 = profile_traffic(name)
        if t1 is None:
            return None
        if world == 1:
            return t1
        return int(round(t1 * per_rank / algorithmic_bytes(M, H, N_glob, wl["res"])))

    traffic_note = ("ncu dram__bytes_read.sum + dram__bytes_write.sum per launch" if world == 1 else
                    f"ncu DRAM bytes of the N=1 capture scaled to this rank's share ({per_rank} of "
                    f"{algorithmic_bytes(M, H, N_glob, wl['res'])} algorithmic bytes)")
    if sched["schedule"] == _lib.SCHED_PREFILL:
        # Tensor-bound: FLOPs of the step over its time (pre-pass + GEMM), against the
        # measured cuBLAS bf16 burst peak.
        gemm = "gemm_pair_kernel (2-CTA tcgen05)" if sched["block_m"] == 256 else "gemm_kernel (tcgen05)"
        achieved = 2.0 * M * N_loc * H / step_s / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / peaks["bf16_tflops"], 4),
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json bf16_tflops, cuBLAS burst)",
                "traffic": traffic(f"prefill_gemm_pair_llama3-8b_m{M}"), "traffic_source": traffic_note,
                "kernel": f"norm_prepass_kernel + {gemm}; time of the whole step"}
    else:
        achieved = per_rank / step_s / 1e9
        kernel = {_lib.SCHED_DECODE: "decode_kernel (fused swap-AB tcgen05, cluster split-K)",
                  _lib.SCHED_GRID: "decode_kernel GRID variant (fused swap-AB tcgen05, K split over CTAs)",
                  _lib.SCHED_SPLIT: "norm_prepass_kernel + streamk_kernel; time of the whole step"}.get(
                      sched["schedule"], "simt_kernel")
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4),
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs, copy burst)",
                "pct_of_8TBs_spec": round(100 * achieved / HBM_SPEC_GBS, 2),
                "traffic": traffic(f"decode_llama3-8b_m{M}")
                if sched["schedule"] in (_lib.SCHED_DECODE, _lib.SCHED_GRID) else None,
                "traffic_source": traffic_note, "kernel": kernel}

    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 6),
        "us_per_step": round(ms_max / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) x/residual, 1+0.1N(0,1) gain, N(0,0.02) weights), random-init",
        "config": {"workload": f"{args.workload} M={M}" + (f" head-sharded over {world} GPUs" if world > 1 else ""),
                   "H": H, "n_q_heads": wl["n_q"], "n_kv_heads": wl["n_kv"], "head_dim": wl["d"],
                   "N_OUT": N_glob, "N_OUT_per_gpu": N_loc, "M": M, "has_residual": wl["res"],
                   "residual_out": True, "weight_sets": wl["sets"],
                   "l2": f"{wl['sets']} rotating weight sets ({wl['sets'] * N_loc * H * 2 / 1e9:.2f} GB per GPU) "
                         f"> 126 MB L2",
                   "parallelism": f"tp{world} (column-parallel by heads)" if world > 1 else "single GPU",
                   "timing": f"K steps in one CUDA graph, replayed {tstats['replays']} times with CUDA events per "
                             f"replay; median replay, max over ranks",
                   "replays": tstats["replays"],
                   "replay_ms": {k: round(v, 6) for k, v in tstats.items() if k.endswith("_ms")},
                   "schedule": {k: v for k, v in sched.items()}},
        "gpu_launches": launches,
        "clocks": sampler.summary(),
        "roofline": roof,
        "e2e": e2e,
        "cpu_baseline": cpu,
    }
    if detail:
        line["detail"] = detail
    if check:
        line["shard_check"] = check
    if pg is not None:
        pg.destroy_process_group()
    return line


def run_profile_case(args) -> int:
    """``--profile-case``: a small fixed workload of the fused op for a profiler capture.

    Seeded x / residual ~ N(0, 1), gains 1 + 0.1 N(0, 1) and weights N(0, 0.02) on cuda:0;
    ``--calls`` eager calls of ``fused_add_rmsnorm_matmul`` (or, with ``--fp8w``,
    ``fused_add_rmsnorm_matmul_fp8w`` on weights quantised by ``quantize_weight_e4m3``)
    rotate over ``--sets`` weight sets (default 4), so that with weights larger than a
    quarter of L2 each captured launch reads its weight from HBM.  Prints one line with a
    checksum of the last output.  No timing is printed: numbers taken under a profiler are
    not benchmark values."""
    from triton_fused_rmsnorm_qkv import (fused_add_rmsnorm_matmul, fused_add_rmsnorm_matmul_fp8w,
                                          quantize_weight_e4m3)

    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    dev = torch.device("cuda", 0)
    H, N, M, n_sets = args.H, args.N, args.m or 16, args.sets or 4
    g = torch.Generator(device=dev).manual_seed(5)
    sets = []
    for _ in range(n_sets):
        gain = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(dt)
        w = (0.02 * torch.randn(N, H, generator=g, device=dev)).to(dt)
        sets.append((gain, quantize_weight_e4m3(w) if args.fp8w else w))
    x = torch.randn(1, M, H, generator=g, device=dev).to(dt)
    r = torch.randn(1, M, H, generator=g, device=dev).to(dt)
    out = None
    for i in range(args.calls):
        gain, w = sets[i % n_sets]
        if args.fp8w:
            out, _ = fused_add_rmsnorm_matmul_fp8w(x, r, gain, w[0], w[1], 1e-5, static_weights=True)
        else:
            out, _ = fused_add_rmsnorm_matmul(x, r, gain, w, 1e-5, schedule=args.schedule, static_weights=True)
    torch.cuda.synchronize()
    print(f"ok M={M} H={H} N={N} calls={args.calls} checksum={float(out.float().abs().sum()):.6e}")
    return 0


def main() -> int:
    ap = argparse.ArgumentParser(description="fused RMSNorm+QKV benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="llama3-8b-decode")
    ap.add_argument("--m", type=int, default=None, help="override the token count M")
    ap.add_argument("--no-detail", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--triton-comparator", choices=("autotune", "fixed", "off"), default="autotune",
                    help="the reference's Triton kernels as a detail comparator (from baseline/_ref)")
    ap.add_argument("--sets", type=int, default=None,
                    help="rotating weight sets (default: the workload's; fewer only for profiling captures)")
    prof = ap.add_argument_group("profiler workload (--profile-case)")
    prof.add_argument("--profile-case", action="store_true",
                      help="run a small fixed workload for an ncu capture instead of the benchmark")
    prof.add_argument("--H", type=int, default=4096)
    prof.add_argument("--N", type=int, default=6144)
    prof.add_argument("--schedule", default=None, help="auto (default), decode, grid, split, prefill or simt")
    prof.add_argument("--dtype", choices=("bf16", "fp16"), default="bf16")
    prof.add_argument("--fp8w", action="store_true", help="e4m3 weights with an fp32 scale per row")
    prof.add_argument("--calls", type=int, default=8)
    args = ap.parse_args()
    if args.profile_case:
        return run_profile_case(args)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    wl = dict(WORKLOADS[args.workload])
    if args.sets:
        wl["sets"] = args.sets
    M = args.m or wl["M"]
    world, rank, _ = dist_env()
    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args, wl, M)), flush=True)
        return 0
    line = run_ours(args, wl, M)
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
