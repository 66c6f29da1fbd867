"""Benchmark suite over the ops (API of the reference's BenchmarkSuite), timed with CUDA events."""

from typing import Callable, List, Optional, Tuple

import torch

from triton_ops.autotuner.tuner import compute_elementwise_metrics, compute_gemm_metrics
from triton_ops.benchmark.correctness import CorrectnessVerifier
from triton_ops.benchmark.report import BenchmarkResult, ComparisonResult, PerformanceReport
from triton_ops.models import KernelMetrics


class BenchmarkSuite:
    def __init__(self, warmup_runs: int = 10, benchmark_runs: int = 100, rtol: float = 1e-3, atol: float = 1e-5):
        self.warmup_runs = warmup_runs
        self.benchmark_runs = benchmark_runs
        self.verifier = CorrectnessVerifier(rtol=rtol, atol=atol)
        self.report = PerformanceReport()
        if torch.cuda.is_available():
            self.report.set_metadata("device", torch.cuda.get_device_name())
            self.report.set_metadata("cuda_version", torch.version.cuda)
        self.report.set_metadata("pytorch_version", torch.__version__)

    def _time_kernel(self, fn: Callable, *args, **kwargs) -> float:
        """Mean milliseconds per call, CUDA events on the current stream."""
        for _ in range(self.warmup_runs):
            fn(*args, **kwargs)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record()
        for _ in range(self.benchmark_runs):
            fn(*args, **kwargs)
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / max(self.benchmark_runs, 1)

    def benchmark_kernel(self, kernel_fn: Callable, reference_fn: Callable, kernel_name: str, problem_size: tuple,
                         inputs: tuple, config: Optional[dict] = None,
                         metrics_fn: Optional[Callable[[tuple, float], KernelMetrics]] = None) -> BenchmarkResult:
        out = kernel_fn(*inputs)
        ref = reference_fn(*inputs)
        ok, _ = self.verifier.verify(out, ref)
        ms = self._time_kernel(kernel_fn, *inputs)
        metrics = metrics_fn(problem_size, ms) if metrics_fn else KernelMetrics(ms, 0.0, 0.0, 0.0)
        result = BenchmarkResult(kernel_name, problem_size, config or {}, metrics, ok)
        self.report.add_result(result)
        return result

    def compare_with_pytorch(self, kernel_fn: Callable, pytorch_fn: Callable, kernel_name: str, problem_size: tuple,
                             inputs: tuple, metrics_fn=None) -> ComparisonResult:
        ok, _ = self.verifier.verify(kernel_fn(*inputs), pytorch_fn(*inputs))
        t_k = self._time_kernel(kernel_fn, *inputs)
        t_b = self._time_kernel(pytorch_fn, *inputs)
        mk = metrics_fn(problem_size, t_k) if metrics_fn else KernelMetrics(t_k, 0.0, 0.0, 0.0)
        mb = metrics_fn(problem_size, t_b) if metrics_fn else KernelMetrics(t_b, 0.0, 0.0, 0.0)
        cmp = ComparisonResult(kernel_name, problem_size, mk, mb, t_b / t_k if t_k > 0 else 0.0, ok)
        self.report.add_comparison(cmp)
        return cmp

    def benchmark_rmsnorm_rope(self, batch_sizes: List[int] = (1, 8), seq_lens: List[int] = (128, 2048),
                               hidden_dims: List[int] = (4096,), head_dim: int = 64,
                               dtype: torch.dtype = torch.float16) -> List[BenchmarkResult]:
        from triton_ops.kernels.rmsnorm_rope import fused_rmsnorm_rope, fused_rmsnorm_rope_reference

        results = []
        for b in batch_sizes:
            for s in seq_lens:
                for h in hidden_dims:
                    x = torch.randn(b, s, h, device="cuda", dtype=dtype)
                    w = torch.ones(h, device="cuda", dtype=dtype)
                    cos = torch.randn(s, head_dim, device="cuda", dtype=dtype)
                    sin = torch.randn(s, head_dim, device="cuda", dtype=dtype)
                    nbytes = 2 * x.element_size()
                    results.append(self.benchmark_kernel(
                        fused_rmsnorm_rope, fused_rmsnorm_rope_reference, "fused_rmsnorm_rope", (b, s, h, head_dim),
                        (x, w, cos, sin),
                        metrics_fn=lambda size, ms, n=x.numel(), bpe=nbytes: compute_elementwise_metrics(n, ms, bpe)))
        return results

    def benchmark_gated_mlp(self, batch_sizes: List[int] = (2,), seq_lens: List[int] = (1024,),
                            hidden_dims: List[int] = (4096,), intermediate_dims: List[int] = (11264,),
                            activation: str = "silu", dtype: torch.dtype = torch.float16) -> List[BenchmarkResult]:
        from triton_ops.kernels.gated_mlp import fused_gated_mlp, gated_mlp_reference

        results = []
        for b in batch_sizes:
            for s in seq_lens:
                for h in hidden_dims:
                    for i in intermediate_dims:
                        x = torch.randn(b, s, h, device="cuda", dtype=dtype)
                        wg = torch.randn(i, h, device="cuda", dtype=dtype) * 0.02
                        wu = torch.randn(i, h, device="cuda", dtype=dtype) * 0.02
                        # two GEMMs per call: 4*M*N*K flops
                        results.append(self.benchmark_kernel(
                            lambda a, g, u: fused_gated_mlp(a, g, u, activation),
                            lambda a, g, u: gated_mlp_reference(a, g, u, activation),
                            "fused_gated_mlp", (b * s, i, h), (x, wg, wu),
                            metrics_fn=lambda size, ms: compute_gemm_metrics(size[0], 2 * size[1], size[2], ms)))
        return results

    def benchmark_fp8_gemm(self, sizes: List[Tuple[int, int, int]] = ((1024, 4096, 4096),)) -> List[BenchmarkResult]:
        from triton_ops.kernels.fp8_gemm import fp8_gemm, fp8_gemm_reference
        from triton_ops.kernels.fp8_quantize import quantize_fp8

        results = []
        for (m, n, k) in sizes:
            a, sa = quantize_fp8(torch.randn(m, k, device="cuda", dtype=torch.float16))
            b, sb = quantize_fp8(torch.randn(k, n, device="cuda", dtype=torch.float16))
            results.append(self.benchmark_kernel(
                fp8_gemm, fp8_gemm_reference, "fp8_gemm", (m, n, k), (a, b, sa, sb),
                metrics_fn=lambda size, ms: compute_gemm_metrics(*size, ms, peak_tflops=4500.0, dtype_bytes=1)))
        return results

    def generate_report(self, format: str = "text") -> str:
        return self.report.generate_json_report() if format == "json" else self.report.generate_text_report()

    def save_report(self, filepath: str, format: str = "text") -> None:
        self.report.save(filepath, format)
