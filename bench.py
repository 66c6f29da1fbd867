"""Benchmark of the fused transformer-op hot path on B200.

Workload (one "step"): the prefill slab of a transformer layer's fused ops,
x [8, 8192, 4096] fp16 (65,536 token rows, N(0, 1)) ->
``fused_rmsnorm_rope`` (weight N(1, 0.1), head_dim 64, RoPE base 10000) ->
``fused_gated_mlp`` (SiLU, gate/up weights [11264, 4096] N(0, 0.02)).
With ``--gpus N`` the 65,536 rows are split into N contiguous slabs, one per
rank (strong scaling); the weights are broadcast once over NCCL at setup and
the timed step has no collective.

Printed (rank 0, one JSON line): ``value`` = whole-job throughput of the step
in TFLOP/s, counting the gated MLP's 4*M*N*K tensor flops (RMSNorm+RoPE adds
no tensor flops but its time is inside the step); ``e2e`` = the same with
pinned-host inputs copied in and the output copied out every step; the
roofline of the dominant kernel (the gated MLP) and of RMSNorm+RoPE from
CUDA events on the launching stream; per-op ``components`` (FP8 codec GB/s,
FP8 GEMM TFLOP/s over M, RMSNorm+RoPE GB/s at the small shape) on rank 0;
SM clocks sampled during the timed region; and the CPU baseline (the numpy
restatement of the reference's PyTorch path, on a bounded row sample).

``--impl reference`` times that CPU path alone (all host threads, bounded row
sample per step) and prints the same metric.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "triton-fused-ops_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "RMSNorm+RoPE HBM GB/s; FP8 GEMM & gated-MLP TFLOPS vs B200 peak"
B, S, H, D, I = 8, 8192, 4096, 64, 11264
ROWS = B * S
FLOPS_PER_ROW = 4 * I * H  # gate + up projections, 2 flops per multiply-add
RMS_BYTES_PER_ROW = 2 * H * 2  # read x + write y (fp16); weight and tables are reused across rows
L2_BYTES = 126 * 2**20


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[4:]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for n, v in zip(names, r[3][1:]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        loaded = [r for r in rows if r[2] > 300] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
def dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def rope_tables(seq_len: int, head_dim: int, device):
    """HF-style cos/sin [seq_len, head_dim] = cat(f, f), f = pos * 10000^(-2i/head_dim), as fp16 on `device`."""
    import torch

    inv = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    f = torch.outer(torch.arange(seq_len, dtype=torch.float64), inv)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().float().half().to(device), emb.sin().float().half().to(device)


def flush_l2(buf):
    buf.add_(1)


def time_events(fn, reps, flush_buf=None):
    """Mean ms of fn() over reps, each timed alone with CUDA events (L2 flushed between reps)."""
    import torch

    st = torch.cuda.current_stream()
    fn()  # first launch loads the kernel's module (lazy loading); not timed
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        if flush_buf is not None:
            flush_l2(flush_buf)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(st)
        fn()
        b.record(st)
        b.synchronize()
        times.append(a.elapsed_time(b))
    return sum(times) / len(times)


# ---------------------------------------------------------------------------
# CPU baseline: the reference's PyTorch CPU path
# ---------------------------------------------------------------------------
# The reference's own CPU implementation of these ops is its PyTorch oracle
# functions (rmsnorm_rope.py:356-383, fp8_quantize.py:258-312,
# fp8_gemm.py:190-225, gated_mlp.py:221-251). This package carries the same
# torch expressions as ``triton_ops.kernels.*.*_reference`` (the reference's
# tests import them); they run here on CPU tensors with every host thread.
CPU_SAMPLE_ROWS = 1024  # token rows per CPU step (positions 0..1023 of one sequence)


def cpu_cores():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def cpu_threads():
    import torch

    torch.set_num_threads(cpu_cores())
    return torch.get_num_threads()


class CpuPath:
    """The prefill step on CPU_SAMPLE_ROWS token rows through the reference's
    PyTorch functions: RMSNorm+RoPE (fp32 math, fp16 result) then the gated MLP
    (fp32 projections of the fp16 operands, SiLU, fp16 result)."""

    def __init__(self, rows: int = CPU_SAMPLE_ROWS):
        import torch

        from triton_ops.kernels.gated_mlp import gated_mlp_reference
        from triton_ops.kernels.rmsnorm_rope import fused_rmsnorm_rope_reference

        self.rows = rows
        self.rms, self.mlp = fused_rmsnorm_rope_reference, gated_mlp_reference
        g = torch.Generator().manual_seed(0)
        self.x = torch.randn(1, rows, H, generator=g).half()
        self.w = (1 + 0.1 * torch.randn(H, generator=g)).half()
        self.cos, self.sin = rope_tables(rows, D, "cpu")
        self.wg = (0.02 * torch.randn(I, H, generator=g)).half()
        self.wu = (0.02 * torch.randn(I, H, generator=g)).half()

    def step(self):
        y = self.rms(self.x, self.w, self.cos, self.sin, 1e-6)
        return self.mlp(y, self.wg, self.wu, "silu")


def cpu_sample_text(rows, n, dt):
    return (f"{rows} of {ROWS} token rows per step (positions 0..{rows - 1}): the reference's PyTorch "
            f"fused_rmsnorm_rope_reference -> gated_mlp_reference (fp32 math) on CPU tensors, "
            f"{n} steps of {dt * 1e3:.1f} ms measured")


def cpu_baseline(max_seconds: float = 12.0):
    """Times the CPU path on a bounded row sample (reported beside the GPU number)."""
    threads = cpu_threads()
    path = CpuPath()
    path.step()  # warm-up (thread pool, first-touch)
    times = []
    t_end = time.perf_counter() + max_seconds
    while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 20):
        t0 = time.perf_counter()
        path.step()
        times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    return {"value": path.rows * FLOPS_PER_ROW / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
            "cpu_model": cpu_model(), "kind": "port", "ms_per_step": dt * 1e3,
            "sample": cpu_sample_text(path.rows, len(times), dt)}


def time_cpu(fn, max_seconds: float = 3.0, max_reps: int = 5):
    """Median seconds of fn() on the CPU after one warm-up call (bounded by max_seconds)."""
    fn()
    times = []
    t_end = time.perf_counter() + max_seconds
    while not times or (time.perf_counter() < t_end and len(times) < max_reps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times)


def cpu_components():
    """The reference's PyTorch CPU functions at every configuration's shape.

    Returns {component name: microseconds per call}; names match the GPU
    `components` entries they sit beside.
    """
    import torch

    from triton_ops.kernels.fp8_gemm import fp8_gemm_reference
    from triton_ops.kernels.fp8_quantize import fp8_dequantize_reference, fp8_quantize_reference
    from triton_ops.kernels.gated_mlp import gated_mlp_reference
    from triton_ops.kernels.rmsnorm_rope import fused_rmsnorm_rope_reference

    cpu_threads()
    g = torch.Generator().manual_seed(7)
    out = {}
    # config 1: [2, 128, 4096], fp32 on the CPU
    x = torch.randn(2, 128, 4096, generator=g)
    w = 1 + 0.1 * torch.randn(4096, generator=g)
    cos, sin = rope_tables(128, 64, "cpu")
    cos, sin = cos.float(), sin.float()
    out["rmsnorm_rope_2x128x4096"] = 1e6 * time_cpu(lambda: fused_rmsnorm_rope_reference(x, w, cos, sin, 1e-6))
    # config 2: [4096, 4096] fp16 with 0.1% outliers of +-200, dynamic scale
    t = torch.randn(4096, 4096, generator=g).half()
    idx = torch.randperm(t.numel(), generator=g)[: t.numel() // 1000]
    t.view(-1)[idx] = 200.0 * torch.sign(torch.randn(idx.numel(), generator=g)).half()
    out["fp8_quantize_4096x4096"] = 1e6 * time_cpu(lambda: fp8_quantize_reference(t))
    q, s = fp8_quantize_reference(t)
    out["fp8_dequantize_4096x4096"] = 1e6 * time_cpu(lambda: fp8_dequantize_reference(q, s))
    # config 3: codes A [M, 4096], B [4096, 4096], fp16 out
    qb, sb = fp8_quantize_reference(torch.randn(4096, 4096, generator=g).half())
    gemm = {}
    for M in (16, 128, 1024, 4096, 8192):
        qa, sa = fp8_quantize_reference(torch.randn(M, 4096, generator=g).half())
        gemm[str(M)] = 1e6 * time_cpu(lambda: fp8_gemm_reference(qa, qb, sa, sb), max_reps=3)
    out["fp8_gemm_Mx4096x4096"] = gemm
    # config 4: x [2, 1024, 4096] fp16, W [11264, 4096] fp16
    xm = torch.randn(2, 1024, 4096, generator=g).half()
    wg = (0.02 * torch.randn(11264, 4096, generator=g)).half()
    wu = (0.02 * torch.randn(11264, 4096, generator=g)).half()
    for act in ("silu", "gelu", "gelu_tanh"):
        out[f"gated_mlp_2x1024x4096_{act}"] = 1e6 * time_cpu(lambda: gated_mlp_reference(xm, wg, wu, act),
                                                             max_reps=3)
    return out


def bench_config(world: int) -> dict:
    """The workload description both arms print (identical for the same N)."""
    return {
        "workload": "prefill RMSNorm+RoPE -> gated MLP (SiLU), x [8, 8192, 4096] fp16 row-sharded, "
                    "W_gate/W_up [11264, 4096] fp16, head_dim 64",
        "rows": ROWS, "rows_per_rank": -(-ROWS // world), "hidden": H, "intermediate": I, "head_dim": D,
        "parallelism": f"rows{world}" if world > 1 else "single",
        "l2": "inputs larger than L2: two alternating x slabs; per-step traffic > 4x L2",
    }


def run_reference(args):
    """The reference's CPU implementation of the path, rank 0 only.

    Each step runs the prefill step's ops on CPU_SAMPLE_ROWS token rows (a
    bounded sample of the 65,536-row slab) and is timed as it runs; `value` is
    the measured rate (tensor flops of the sample / step time) and
    `ms_per_step` the measured time of one sample step.
    """
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    threads = cpu_threads()
    path = CpuPath()
    for _ in range(args.warmup):
        path.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        path.step()
    dt = (time.perf_counter() - t0) / args.steps
    value = path.rows * FLOPS_PER_ROW / dt / 1e12
    sample = cpu_sample_text(path.rows, args.steps, dt)
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16 (fp32 math on CPU)",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, N(1,0.1) norm weight)",
            "config": bench_config(world),
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "cpu_model": cpu_model(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------
# GPU step
# ---------------------------------------------------------------------------
def time_graph(calls, reps: int = 20):
    """Device-side microseconds per call.

    `calls` hold one call per rotating input set (together larger than L2, so
    each call finds its inputs in HBM). They are captured once into a CUDA
    graph, which is replayed `reps` times between two CUDA events; host work
    per call (Python, validation, ctypes) is outside the measurement.
    Returns (us, None) or (None, error text) if the capture failed.
    """
    import torch

    for c in calls:
        c()  # lazy module loading, workspace sizing
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for c in calls:
            c()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(g):
            for c in calls:
                c()
    except Exception as exc:  # noqa: BLE001 - reported in the JSON line
        torch.cuda.synchronize()
        return None, f"{type(exc).__name__}: {exc}"[:200]
    g.replay()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    b.synchronize()
    us = a.elapsed_time(b) * 1e3 / (reps * len(calls))
    del g
    torch.cuda.synchronize()
    return us, None


def host_us_per_call(fn, calls: int = 200) -> float:
    """Host (CPU) microseconds per call: wall clock over back-to-back calls that
    are not synchronised, so the GPU runs behind and the Python, validation,
    allocation and launch work of each call is what is timed (one warm-up
    round first; the launch queue holds them all)."""
    import torch

    for _ in range(20):
        fn()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(calls):
        fn()
    t1 = time.perf_counter()
    torch.cuda.synchronize()
    return (t1 - t0) * 1e6 / calls


def _copies(make, nbytes_each: int, min_total: int = 2 * L2_BYTES, cap: int = 128):
    """Enough independent tensors from make() that together they exceed min_total bytes."""
    n = max(2, min(cap, -(-min_total // max(1, nbytes_each))))
    return [make() for _ in range(n)]


def components(peaks, flush_buf):
    """Per-op numbers at the other configurations (rank 0).

    For each op: ``us`` = device time per call from CUDA-graph replay over
    rotating inputs larger than L2 (the kernel-side number the roofline
    fraction uses), ``us_call`` = one eager call through the Python API timed
    alone with CUDA events after an L2 flush (device-side: the flush kernel is
    still running when the call's launches are queued, so this adds cold-L2
    inputs and the gaps between eager launches, not host time), and for the
    decode-size calls ``host_us`` = host time per call (see host_us_per_call).
    """
    import torch

    import triton_ops

    out = {}
    dev = torch.device("cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    hbm = peaks["hbm_gbs"]

    def entry(us, err, us_call, nbytes=None, flops=None, peak=None):
        e = {"us": us, "us_call": us_call}
        if err:
            e["graph_error"] = err
        t = us if us is not None else us_call
        if nbytes is not None:
            e["GB/s"] = nbytes / t / 1e3
            e["frac_hbm"] = nbytes / t / 1e3 / hbm
        if flops is not None:
            e["TFLOP/s"] = flops / t / 1e6
            if peak is not None:
                e["frac_peak"] = flops / t / 1e6 / peak
        return e

    # RMSNorm+RoPE at [2, 128, 4096] (launch-latency bound)
    def mk_x():
        return torch.randn(2, 128, 4096, device=dev, dtype=torch.float16, generator=g)
    xs = _copies(mk_x, 2 * 128 * 4096 * 2)
    w = (1 + 0.1 * torch.randn(4096, device=dev, generator=g)).half()
    cos, sin = rope_tables(128, 64, dev)
    nbytes = 2 * (2 * 128 * 4096 * 2) + 4096 * 2 + 2 * (128 * 32 * 2)
    us, err = time_graph([lambda x=x: triton_ops.fused_rmsnorm_rope(x, w, cos, sin) for x in xs])
    us_call = 1e3 * time_events(lambda: triton_ops.fused_rmsnorm_rope(xs[0], w, cos, sin), 50, flush_buf)
    out["rmsnorm_rope_2x128x4096"] = entry(us, err, us_call, nbytes=nbytes)
    del xs

    # FP8 quantize / dequantize at [4096, 4096] fp16 with 0.1% outliers of +-200
    def mk_t():
        t = torch.randn(4096, 4096, device=dev, generator=g).half()
        idx = torch.randperm(t.numel(), device=dev, generator=g)[: t.numel() // 1000]
        t.view(-1)[idx] = 200.0 * torch.sign(torch.randn(idx.numel(), device=dev, generator=g)).half()
        return t
    ts = _copies(mk_t, 4096 * 4096 * 2)
    nb = 3 * 4096 * 4096
    for name, qd in (("", torch.uint8), ("_e4m3", torch.float8_e4m3fn)):
        us, err = time_graph([lambda t=t: triton_ops.quantize_fp8(t, dtype=qd) for t in ts])
        us_call = 1e3 * time_events(lambda: triton_ops.quantize_fp8(ts[0], dtype=qd), 30, flush_buf)
        out[f"fp8_quantize{name}_4096x4096"] = entry(us, err, us_call, nbytes=nb)
        qs = [triton_ops.quantize_fp8(t, dtype=qd) for t in ts]
        us, err = time_graph([lambda q=q, s=s: triton_ops.dequantize_fp8(q, s) for q, s in qs])
        us_call = 1e3 * time_events(lambda: triton_ops.dequantize_fp8(*qs[0]), 30, flush_buf)
        out[f"fp8_dequantize{name}_4096x4096"] = entry(us, err, us_call, nbytes=nb)
        del qs
    del ts

    # decode-size activations: dynamic-scale quantize of [16, 4096] fp16 and
    # FP8Linear(4096 -> 4096, bias) on it (quantize + codec GEMM + bias epilogue)
    xd = [torch.randn(1, 16, 4096, device=dev, generator=g).half() for _ in range(16)]
    us, err = time_graph([lambda x=x: triton_ops.quantize_fp8(x) for x in xd])
    us_call = 1e3 * time_events(lambda: triton_ops.quantize_fp8(xd[0]), 30, flush_buf)
    out["fp8_quantize_16x4096"] = entry(us, err, us_call, nbytes=3 * 16 * 4096)
    out["fp8_quantize_16x4096"]["host_us"] = host_us_per_call(lambda: triton_ops.quantize_fp8(xd[0]))
    lin = triton_ops.FP8Linear(4096, 4096, bias=True).to(dev).half()
    us, err = time_graph([lambda x=x: lin(x) for x in xd])
    us_call = 1e3 * time_events(lambda: lin(xd[0]), 30, flush_buf)
    out["fp8linear_16x4096x4096"] = entry(us, err, us_call, flops=2.0 * 16 * 4096 * 4096)
    out["fp8linear_16x4096x4096"]["host_us"] = host_us_per_call(lambda: lin(xd[0]))
    out["native_extension_loaded"] = _lib_ext_loaded()
    del xd, lin

    # per-token scales at [4096, 4096] fp16: the row scales, then quantize and
    # dequantize with one scale per row (reference codec)
    xr = _copies(lambda: torch.randn(4096, 4096, device=dev, generator=g).half(), 4096 * 4096 * 2)
    per_row = triton_ops.FP8Format.compute_scale_per_channel
    rs = [per_row(x, dim=-1).float() for x in xr]
    us, err = time_graph([lambda x=x: per_row(x, dim=-1) for x in xr])
    us_call = 1e3 * time_events(lambda: per_row(xr[0], dim=-1), 30, flush_buf)
    out["fp8_row_scales_4096x4096"] = entry(us, err, us_call, nbytes=2 * 4096 * 4096)
    us, err = time_graph([lambda x=x, s=s: triton_ops.quantize_fp8(x, s) for x, s in zip(xr, rs)])
    us_call = 1e3 * time_events(lambda: triton_ops.quantize_fp8(xr[0], rs[0]), 30, flush_buf)
    out["fp8_quantize_rows_4096x4096"] = entry(us, err, us_call, nbytes=3 * 4096 * 4096)
    # per-token dynamic quantize in one launch, against the two calls it replaces
    us, err = time_graph([lambda x=x: triton_ops.quantize_fp8_per_token(x) for x in xr])
    us_call = 1e3 * time_events(lambda: triton_ops.quantize_fp8_per_token(xr[0]), 30, flush_buf)
    e = entry(us, err, us_call, nbytes=3 * 4096 * 4096)
    e["two_calls_us"], _ = time_graph([lambda x=x: triton_ops.quantize_fp8(x, per_row(x, dim=-1)) for x in xr])
    out["fp8_quantize_per_token_4096x4096"] = e
    qr = [triton_ops.quantize_fp8(x, s)[0] for x, s in zip(xr, rs)]
    del xr
    us, err = time_graph([lambda q=q, s=s: triton_ops.dequantize_fp8(q, s) for q, s in zip(qr, rs)])
    us_call = 1e3 * time_events(lambda: triton_ops.dequantize_fp8(qr[0], rs[0]), 30, flush_buf)
    out["fp8_dequantize_rows_4096x4096"] = entry(us, err, us_call, nbytes=3 * 4096 * 4096)
    del qr, rs

    # FP8 GEMM over M, N = K = 4096: reference codec (int8 tensor cores), e4m3
    # (fp8 tensor cores), and the library fp8 GEMM (torch._scaled_mm) on the
    # same e4m3 operands as a comparator
    def mk_b():
        return torch.randn(4096, 4096, device=dev, generator=g).half()
    bs = [triton_ops.quantize_fp8(b, dtype=torch.uint8) for b in _copies(mk_b, 4096 * 4096, cap=16)]
    bs8 = [triton_ops.quantize_fp8(b, dtype=torch.float8_e4m3fn) for b in _copies(mk_b, 4096 * 4096, cap=16)]
    bs8_nk = [(q.t().contiguous(), s) for q, s in bs8]
    gemm, gemm8, lib8 = {}, {}, {}
    for M in (16, 128, 1024, 4096, 8192):
        fl = 2.0 * M * 4096 * 4096
        def mk_a():
            return torch.randn(M, 4096, device=dev, generator=g).half()
        a_f = _copies(mk_a, M * 4096, cap=len(bs))
        a_f = (a_f * ((len(bs) + len(a_f) - 1) // len(a_f)))[: len(bs)]
        qa = [triton_ops.quantize_fp8(a, dtype=torch.uint8) for a in a_f]
        qa8 = [triton_ops.quantize_fp8(a, dtype=torch.float8_e4m3fn) for a in a_f]
        pairs = list(zip(qa, bs))
        us, err = time_graph([lambda a=a, b=b: triton_ops.fp8_gemm(a[0], b[0], a[1], b[1]) for a, b in pairs])
        us_call = 1e3 * time_events(lambda: triton_ops.fp8_gemm(qa[0][0], bs[0][0], qa[0][1], bs[0][1]), 20, flush_buf)
        gemm[str(M)] = entry(us, err, us_call, flops=fl)
        pairs8 = list(zip(qa8, bs8))
        us, err = time_graph([lambda a=a, b=b: triton_ops.fp8_gemm(a[0], b[0], a[1], b[1]) for a, b in pairs8])
        us_call = 1e3 * time_events(lambda: triton_ops.fp8_gemm(qa8[0][0], bs8[0][0], qa8[0][1], bs8[0][1]), 20,
                                    flush_buf)
        gemm8[str(M)] = entry(us, err, us_call, flops=fl)
        try:
            one = torch.ones((), device=dev)
            libs = [lambda a=a, b=b: torch._scaled_mm(a[0], b[0].t(), one, one, out_dtype=torch.float16)
                    for a, b in zip(qa8, bs8_nk)]
            us, err = time_graph(libs)
            lib8[str(M)] = entry(us, err, None, flops=fl)
        except Exception as exc:  # noqa: BLE001 - comparator only
            lib8[str(M)] = {"error": f"{type(exc).__name__}: {exc}"[:200]}
        del qa, qa8, a_f
    # the same products with B given as [N, K] (K-major: FP8Linear's weight
    # layout, and the layout of the cuBLASLt comparator above), small M
    from triton_ops.kernels.fp8_gemm import _gemm_codes
    from triton_ops import _lib as tfo_lib
    bs_nk = [(q.t().contiguous(), s_) for q, s_ in bs]
    gemm_nk, gemm8_nk = {}, {}
    for M in (16, 32, 128, 1024):
        fl = 2.0 * M * 4096 * 4096
        a_f = _copies(lambda: torch.randn(M, 4096, device=dev, generator=g).half(), M * 4096, cap=len(bs))
        a_f = (a_f * ((len(bs) + len(a_f) - 1) // len(a_f)))[: len(bs)]
        for table, qd, bl in ((gemm_nk, torch.uint8, bs_nk), (gemm8_nk, torch.float8_e4m3fn, bs8_nk)):
            qa = [triton_ops.quantize_fp8(a, dtype=qd) for a in a_f]
            us, err = time_graph([lambda a=a, b=b: _gemm_codes(a[0], b[0], a[1], b[1], torch.float16, tfo_lib.B_NK)
                                  for a, b in zip(qa, bl)])
            e = entry(us, err, None, flops=fl)
            if us is not None and M <= 128:
                nbytes = M * 4096 + 4096 * 4096 + 2 * M * 4096
                ach = nbytes / us / 1e3
                e["roofline"] = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                                 "algorithmic_bytes": nbytes, "peak_source": f"{peaks['source']} hbm_gbs"}
            table[str(M)] = e
        del a_f
    out["fp8_gemm_nk_Mx4096x4096"] = gemm_nk
    out["fp8_gemm_nk_e4m3_Mx4096x4096"] = gemm8_nk
    del bs, bs8, bs8_nk, bs_nk
    # FP8 tensor peak measured in this run: the library fp8 GEMM (cuBLASLt
    # through torch._scaled_mm, e4m3, fp32 accumulate) at 8192^3, best of 10
    # back-to-back launches (a burst, like the bf16 peak); 2 x the measured
    # bf16 burst is reported beside it
    fp8_peak = None
    try:
        pa = torch.randn(8192, 8192, device=dev, generator=g).to(torch.float8_e4m3fn)
        pb = torch.randn(8192, 8192, device=dev, generator=g).to(torch.float8_e4m3fn)
        one = torch.ones((), device=dev)
        best = min(time_events(lambda: torch._scaled_mm(pa, pb.t(), one, one, out_dtype=torch.bfloat16), 1)
                   for _ in range(10))
        fp8_peak = 2.0 * 8192**3 / (best / 1e3) / 1e12
        del pa, pb
    except Exception as exc:  # noqa: BLE001 - reported as missing
        out["fp8_peak_error"] = f"{type(exc).__name__}: {exc}"[:200]
    out["fp8_tensor_peak"] = {"TFLOP/s": fp8_peak, "how": "torch._scaled_mm e4m3 8192^3 -> bf16, best of 10, "
                                                          "CUDA events, in this run",
                              "two_x_bf16_burst": 2 * peaks["bf16_tflops"]}
    for table in (gemm, gemm8):
        for m, e in table.items():
            M = int(m)
            if e.get("us") is None:
                continue
            if M <= 128:  # below the ridge: bound by the operand bytes
                nbytes = M * 4096 + 4096 * 4096 + 2 * M * 4096
                ach = nbytes / e["us"] / 1e3
                e["roofline"] = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                                 "algorithmic_bytes": nbytes, "peak_source": f"{peaks['source']} hbm_gbs"}
            elif fp8_peak:
                e["roofline"] = {"bound": "tensor", "achieved": e["TFLOP/s"], "peak": fp8_peak, "unit": "TFLOP/s",
                                 "frac": e["TFLOP/s"] / fp8_peak,
                                 "peak_source": "fp8 library GEMM measured in this run (fp8_tensor_peak)",
                                 "frac_of_2x_bf16_burst": e["TFLOP/s"] / (2 * peaks["bf16_tflops"])}
    out["fp8_gemm_Mx4096x4096"] = gemm
    out["fp8_gemm_e4m3_Mx4096x4096"] = gemm8
    out["library_scaled_mm_e4m3_Mx4096x4096"] = lib8

    # fused RMSNorm+RoPE -> 8-bit codes at the prefill shape [8, 8192, 4096] fp16,
    # dynamic and given scale, and the two ops run separately; GB/s counts the
    # op's own input and output (8 KB of x read + 4 KB of codes written per row)
    xq = [torch.randn(8, 8192, 4096, device=dev, generator=g).half() for _ in range(2)]
    wq = (1 + 0.1 * torch.randn(4096, device=dev, generator=g)).half()
    cq, sq = rope_tables(8192, 64, dev)
    rows = 8 * 8192
    two = torch.tensor(2.0, device=dev)
    # RMSNorm+RoPE alone at the same shape, two alternating 512 MB inputs (each
    # call starts with its input out of L2): the kernel's own HBM rate. The
    # step's roofline_rmsnorm_rope figure also pays for writing the previous
    # step's gated-MLP output back from L2 while the kernel runs.
    us, err = time_graph([lambda x=x: triton_ops.fused_rmsnorm_rope(x, wq, cq, sq) for x in xq], reps=5)
    out["rmsnorm_rope_8x8192x4096"] = entry(us, err, None, nbytes=rows * RMS_BYTES_PER_ROW + 4096 * 2 + 2 * 8192 * 32 * 2)
    fq = {}
    us, err = time_graph([lambda x=x: triton_ops.fused_rmsnorm_rope_quantize(x, wq, cq, sq) for x in xq], reps=5)
    fq["dynamic_scale"] = entry(us, err, None, nbytes=rows * (8192 + 4096))
    us, err = time_graph([lambda x=x: triton_ops.fused_rmsnorm_rope_quantize(x, wq, cq, sq, scale=two) for x in xq],
                         reps=5)
    fq["given_scale"] = entry(us, err, None, nbytes=rows * (8192 + 4096))
    us, err = time_graph([lambda x=x: triton_ops.quantize_fp8(triton_ops.fused_rmsnorm_rope(x, wq, cq, sq))
                          for x in xq], reps=5)
    fq["unfused_dynamic"] = {"us": us, "graph_error": err}
    us, err = time_graph([lambda x=x: triton_ops.quantize_fp8(triton_ops.fused_rmsnorm_rope(x, wq, cq, sq), two)
                          for x in xq], reps=5)
    fq["unfused_given_scale"] = {"us": us, "graph_error": err}
    out["rmsnorm_rope_quantize_8x8192x4096"] = fq
    del xq

    # gated MLP at [2, 1024, 4096] x [11264, 4096] (weights alone exceed L2)
    xm = [torch.randn(2, 1024, 4096, device=dev, generator=g).half() for _ in range(2)]
    wg = (0.02 * torch.randn(11264, 4096, device=dev, generator=g)).half()
    wu = (0.02 * torch.randn(11264, 4096, device=dev, generator=g)).half()
    fl = 4.0 * 2048 * 11264 * 4096
    for act in ("silu", "gelu", "gelu_tanh"):
        us, err = time_graph([lambda x=x: triton_ops.fused_gated_mlp(x, wg, wu, act) for x in xm], reps=10)
        us_call = 1e3 * time_events(lambda: triton_ops.fused_gated_mlp(xm[0], wg, wu, act), 20, flush_buf)
        out[f"gated_mlp_2x1024x4096_{act}"] = entry(us, err, us_call, flops=fl, peak=peaks["bf16_tflops"])
    # the same MLP with 8-bit output codes (given / dynamic scale) against the two ops
    sc = torch.tensor(40.0, device=dev)
    mq = {}
    us, err = time_graph([lambda x=x: triton_ops.fused_gated_mlp_quantize(x, wg, wu, "silu", sc) for x in xm], reps=10)
    mq["given_scale"] = entry(us, err, None, flops=fl, peak=peaks["bf16_tflops"])
    us, err = time_graph([lambda x=x: triton_ops.fused_gated_mlp_quantize(x, wg, wu, "silu") for x in xm], reps=10)
    mq["dynamic_scale"] = entry(us, err, None, flops=fl, peak=peaks["bf16_tflops"])
    us, err = time_graph([lambda x=x: triton_ops.quantize_fp8(triton_ops.fused_gated_mlp(x, wg, wu, "silu"), sc)
                          for x in xm], reps=10)
    mq["unfused_given_scale"] = entry(us, err, None, flops=fl, peak=peaks["bf16_tflops"])
    out["gated_mlp_quantize_2x1024x4096_silu"] = mq
    return out


def add_cpu_numbers(comps, cpu, threads):
    """Puts each CPU time beside the GPU component of the same name."""
    kind = f"port: the reference's PyTorch function on CPU tensors, {threads} threads"
    for name, v in cpu.items():
        target = comps.get(name)
        if target is None:
            continue
        pairs = v.items() if isinstance(v, dict) else [(None, v)]
        for key, cpu_us in pairs:
            e = target.get(key) if key is not None else target
            if not isinstance(e, dict):
                continue
            e["cpu_us"] = cpu_us
            e["cpu_kind"] = kind + (" (fp32 input)" if name == "rmsnorm_rope_2x128x4096" else "")
            if e.get("us"):
                e["gpu_speedup_vs_cpu"] = cpu_us / e["us"]


def _lib_ext_loaded() -> bool:
    from triton_ops import _lib

    return _lib.ext() is not None


def read_traffic():
    """DRAM bytes per launch of the gated-MLP kernel from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "gated_mlp_prefill_ncu.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_full_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


E2E_CHUNK_ROWS = 4096  # rows per pipelined chunk; divides every slab and every sequence


def run_e2e(args, world, rank, shard, w, wg, wu, cos, sin, x_dev, total_flops):
    """The step through the public API with the input copied from pinned host
    memory and the output copied back to pinned host memory, every step.

    Each rank's slab is processed in chunks of E2E_CHUNK_ROWS rows (each inside
    one sequence, so its RoPE rows are a contiguous slice of the tables) on
    three streams: host->device copy of chunk i+1, RMSNorm+RoPE -> gated MLP of
    chunk i and device->host copy of chunk i-1 overlap. Two device input
    buffers; output tensors come from the caching allocator and are kept
    alive for the copy stream with record_stream.
    """
    import torch

    import triton_ops

    rows = shard.rows
    cr = E2E_CHUNK_ROWS if rows % E2E_CHUNK_ROWS == 0 else rows
    nchunks = rows // cr
    hx = torch.empty(rows, H, dtype=torch.float16, pin_memory=True)
    hx.copy_(x_dev.reshape(rows, H).cpu())
    hout = torch.empty(rows, I, dtype=torch.float16, pin_memory=True)
    dev = x_dev.device
    dx = [torch.empty(1, cr, H, dtype=torch.float16, device=dev) for _ in range(2)]
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    tables = []
    for c in range(nchunks):
        g0 = shard.start + c * cr
        off = g0 % S
        if off + cr <= S:
            tables.append((cos[off:off + cr], sin[off:off + cr]))
        else:  # chunk crosses a sequence boundary (only when a slab is not sequence-aligned)
            pos = torch.arange(g0, g0 + cr, device=dev) % S
            tables.append((cos.index_select(0, pos), sin.index_select(0, pos)))
    main = torch.cuda.current_stream(dev)

    def one_step():
        for c in range(nchunks):
            b = c % 2
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_used[b])
                dx[b].view(cr, H).copy_(hx[c * cr:(c + 1) * cr], non_blocking=True)
                ev_in[b].record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(ev_in[b])
                y = triton_ops.fused_rmsnorm_rope(dx[b], w, tables[c][0], tables[c][1])
                ev_used[b].record(s_cmp)
                o = triton_ops.fused_gated_mlp(y, wg, wu, "silu")
                o.record_stream(s_out)
                ev_done[b].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[b])
                hout[c * cr:(c + 1) * cr].copy_(o.view(cr, I), non_blocking=True)

    def join():
        for s_ in (s_in, s_cmp, s_out):
            main.wait_stream(s_)

    for s_ in (s_in, s_cmp, s_out):
        s_.wait_stream(main)
    for _ in range(max(1, args.warmup // 2)):
        one_step()
    join()
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(main)
    for s_ in (s_in, s_cmp, s_out):
        s_.wait_stream(main)
    for _ in range(args.steps):
        one_step()
    join()
    e1.record(main)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    return {"value": total_flops / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": ROWS * H * 2, "d2h_bytes_per_step": ROWS * I * 2,
            "ms_per_step": e2e_ms / args.steps,
            "pipeline": f"{nchunks} chunks of {cr} rows per rank; H2D, compute and D2H on three streams"}


def run_ours(args):
    import torch

    import triton_ops
    from triton_ops import _lib
    from triton_ops.sharding import broadcast_tensors, shard_rows, slab_tables

    rank, world, local = dist_setup()
    dev = torch.device("cuda", local)
    peaks = measured_peaks()
    shard = shard_rows(ROWS, world, rank)
    rows = shard.rows

    # weights + tables: made on rank 0, broadcast once (setup, untimed)
    g = torch.Generator(device=dev).manual_seed(1234)
    wg = (0.02 * torch.randn(I, H, device=dev, generator=g)).half()
    wu = (0.02 * torch.randn(I, H, device=dev, generator=g)).half()
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).half()
    cos, sin = rope_tables(S, D, dev)
    if world > 1:
        broadcast_tensors([wg, wu, w, cos, sin], src=0)
    cos_s, sin_s, nb, sl = slab_tables(cos, sin, shard, S)

    # two input slabs, alternated, so a step never finds its input in L2
    gx = torch.Generator(device=dev).manual_seed(99 + rank)
    xs = [torch.randn(nb, sl, H, device=dev, generator=gx).half() for _ in range(2)]

    def step(i):
        yy = triton_ops.fused_rmsnorm_rope(xs[i % 2], w, cos_s, sin_s)
        return triton_ops.fused_gated_mlp(yy, wg, wu, "silu")

    st = torch.cuda.current_stream()
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    _lib.device_error_flags(clear=True)

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    launches0 = _lib.kernel_launches()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(st)
        for i in range(args.steps):
            ev[i][0].record(st)
            yy = triton_ops.fused_rmsnorm_rope(xs[i % 2], w, cos_s, sin_s)
            ev[i][1].record(st)
            triton_ops.fused_gated_mlp(yy, wg, wu, "silu")
            ev[i][2].record(st)
        t_end.record(st)
        torch.cuda.synchronize()
    barrier(world)
    launches = _lib.kernel_launches() - launches0
    elapsed_ms = t_start.elapsed_time(t_end)
    rms_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps
    mlp_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps
    elapsed_ms = max_over_ranks(elapsed_ms, world)
    rms_ms = max_over_ranks(rms_ms, world)
    mlp_ms = max_over_ranks(mlp_ms, world)
    clk = clocks.summary()
    flags = _lib.device_error_flags(clear=True)

    total_flops = ROWS * FLOPS_PER_ROW * args.steps
    value = total_flops / (elapsed_ms / 1e3) / 1e12
    mlp_flops_launch = rows * FLOPS_PER_ROW
    rms_bytes_launch = rows * RMS_BYTES_PER_ROW + H * 2 + 2 * S * (D // 2) * 2

    # ---- end to end: pinned host input in, host output out, every step ----
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, world, rank, shard, w, wg, wu, cos, sin, xs[0], total_flops)

    comps = None
    cpu = None
    if rank == 0 and world == 1:
        flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=dev)
        if not args.no_components:
            comps = components(peaks, flush)
        if not args.no_cpu_baseline:
            cpu = cpu_baseline()
            if comps is not None:
                add_cpu_numbers(comps, cpu_components(), cpu["cores"])

    if rank == 0:
        mlp_tflops = mlp_flops_launch / (mlp_ms / 1e3) / 1e12
        rms_gbs = rms_bytes_launch / (rms_ms / 1e3) / 1e9
        traffic = read_traffic()
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f16 (fp32 accumulate)",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, N(1,0.1) norm weight)",
            "config": bench_config(world),
            "roofline": {
                "bound": "tensor", "kernel": "gated_mlp (tcgen05 kind::f16)",
                "achieved": mlp_tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": mlp_tflops / peaks["bf16_tflops"],
                "peak_source": f"{peaks['source']} bf16_tflops (burst: the timed region is ~0.1 s at full clocks)",
                "frac_of_sustained_peak": mlp_tflops / peaks["bf16_tflops_sustained"],
                "traffic": traffic,
                "algorithmic_flops_per_launch": mlp_flops_launch,
            },
            "roofline_rmsnorm_rope": {
                "bound": "hbm", "achieved": rms_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": rms_gbs / peaks["hbm_gbs"], "peak_source": f"{peaks['source']} hbm_gbs",
                "algorithmic_bytes_per_launch": rms_bytes_launch, "us_per_launch": rms_ms * 1e3,
            },
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clk,
            "device_error_flags": flags,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if comps is not None:
            line["components"] = comps
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def run_profile_op(args):
    """Runs one op `--steps` times at a named shape (a small program for ncu captures; prints no bench line)."""
    import torch

    import triton_ops

    dev = torch.device("cuda")
    g = torch.Generator(device="cuda").manual_seed(0)
    op, shape = args.profile_op, args.profile_shape
    if op == "gated_mlp":
        m = {"config4": 2048, "prefill": ROWS, "small": 1024}[shape]
        x = torch.randn(1, m, H, device=dev, generator=g).half()
        wg = (0.02 * torch.randn(I, H, device=dev, generator=g)).half()
        wu = (0.02 * torch.randn(I, H, device=dev, generator=g)).half()
        fn = lambda: triton_ops.fused_gated_mlp(x, wg, wu, "silu")
    elif op == "rmsnorm_rope":
        bsz = {"config1": 2, "prefill": 8, "small": 1}[shape]
        seq = 128 if shape == "config1" else S
        x = torch.randn(bsz, seq, H, device=dev, generator=g).half()
        w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).half()
        cos, sin = rope_tables(seq, D, dev)
        fn = lambda: triton_ops.fused_rmsnorm_rope(x, w, cos, sin)
    elif op == "fp8_gemm":
        m = {"m16": 16, "small": 128, "config4": 1024, "config3": 8192, "prefill": 8192}[shape]
        qd = torch.float8_e4m3fn if args.profile_dtype == "e4m3" else torch.uint8
        qa, sa = triton_ops.quantize_fp8(torch.randn(m, H, device=dev, generator=g).half(), dtype=qd)
        qb, sb = triton_ops.quantize_fp8(torch.randn(H, H, device=dev, generator=g).half(), dtype=qd)
        fn = lambda: triton_ops.fp8_gemm(qa, qb, sa, sb)
    elif op in ("rmsnorm_rope_quantize", "rmsnorm_rope_quantize_given", "rmsnorm_rope_then_quantize_given"):
        x = torch.randn(8, S, H, device=dev, generator=g).half()
        w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).half()
        cos, sin = rope_tables(S, D, dev)
        two = torch.tensor(2.0, device=dev)
        if op == "rmsnorm_rope_quantize":
            fn = lambda: triton_ops.fused_rmsnorm_rope_quantize(x, w, cos, sin)
        elif op == "rmsnorm_rope_quantize_given":
            fn = lambda: triton_ops.fused_rmsnorm_rope_quantize(x, w, cos, sin, scale=two)
        else:
            fn = lambda: triton_ops.quantize_fp8(triton_ops.fused_rmsnorm_rope(x, w, cos, sin), two)
    elif op == "quantize_per_token":
        # [4096, 4096] fp16 N(0, 1): per-row scales and codes in one launch
        t = torch.randn(4096, 4096, device=dev, generator=g).half()
        qd = torch.float8_e4m3fn if args.profile_dtype == "e4m3" else torch.uint8
        fn = lambda: triton_ops.quantize_fp8_per_token(t, dtype=qd)
    elif op in ("quantize", "dequantize"):
        # [4096, 4096] fp16 N(0, 1) with 0.1% of entries set to +-200
        t = torch.randn(4096, 4096, device=dev, generator=g).half()
        idx = torch.randperm(t.numel(), device=dev, generator=g)[: t.numel() // 1000]
        t.view(-1)[idx] = 200.0 * torch.sign(torch.randn(idx.numel(), device=dev, generator=g)).half()
        qd = torch.float8_e4m3fn if args.profile_dtype == "e4m3" else torch.uint8
        q, s = triton_ops.quantize_fp8(t, dtype=qd)
        fn = (lambda: triton_ops.quantize_fp8(t, dtype=qd)) if op == "quantize" else (lambda: triton_ops.dequantize_fp8(q, s))
    else:
        raise SystemExit(f"unknown op {op}")
    for _ in range(args.steps):
        fn()
    torch.cuda.synchronize()
    print(json.dumps({"profile_op": op, "shape": shape, "launches": args.steps}))
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-components", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-op", default=None,
                    help="run one op --steps times for an ncu capture: gated_mlp, rmsnorm_rope, fp8_gemm, quantize, "
                         "dequantize, quantize_per_token")
    ap.add_argument("--profile-shape", default="small", help="small | config1 | config3 | config4 | prefill")
    ap.add_argument("--profile-dtype", default="u8", choices=["u8", "e4m3"],
                    help="8-bit code of the fp8_gemm / quantize / dequantize profile runs")
    args = ap.parse_args()
    if args.profile_op:
        return run_profile_op(args)
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
