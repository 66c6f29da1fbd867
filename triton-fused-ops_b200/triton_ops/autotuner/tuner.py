"""Configuration search over a user callable (API of the reference's TritonAutoTuner).

The library's own ops never call this (they use the static tile table); it
times a callable with CUDA events for users who want to search their own
parameters.
"""

from typing import Any, Callable, Dict, List, Optional, Tuple

import torch

from triton_ops.autotuner.cache import ConfigCache
from triton_ops.autotuner.configs import generate_configs
from triton_ops.exceptions import TuningFailedError
from triton_ops.models import KernelMetrics, TuningResult

# B200 peaks used for utilisation figures: measured, not nominal (a cuBLAS bf16
# GEMM at 8192^3, best of 10, and a 1 Gi-element device copy counting read +
# write bytes); the nominal figures are 2250 TFLOP/s dense bf16 and 7.7 TB/s
B200_PEAK_TFLOPS_BF16 = 1690.5
B200_PEAK_HBM_GBPS = 6554.6


class TritonAutoTuner:
    def __init__(self, kernel_fn: Callable, config_space: Dict[str, List[Any]], warmup_runs: int = 10,
                 benchmark_runs: int = 100, cache_dir: Optional[str] = None):
        self.kernel_fn = kernel_fn
        self.config_space = config_space
        self.warmup_runs = warmup_runs
        self.benchmark_runs = benchmark_runs
        self.cache = ConfigCache(cache_dir)
        self.all_configs = generate_configs(config_space)

    def _benchmark_config(self, config: Dict[str, Any], *args, **kwargs) -> Optional[KernelMetrics]:
        try:
            for _ in range(self.warmup_runs):
                self.kernel_fn(*args, **config, **kwargs)
            if torch.cuda.is_available():
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                start.record()
                for _ in range(self.benchmark_runs):
                    self.kernel_fn(*args, **config, **kwargs)
                end.record()
                torch.cuda.synchronize()
                latency_ms = start.elapsed_time(end) / max(self.benchmark_runs, 1)
            else:
                import time

                t0 = time.perf_counter()
                for _ in range(self.benchmark_runs):
                    self.kernel_fn(*args, **config, **kwargs)
                latency_ms = (time.perf_counter() - t0) * 1e3 / max(self.benchmark_runs, 1)
            return KernelMetrics(latency_ms=latency_ms, throughput_tflops=0.0, bandwidth_gbps=0.0,
                                 bandwidth_utilization=0.0)
        except Exception:
            return None

    def tune(self, *args, problem_size: Tuple[int, ...] = None, device: str = None, kernel_type: str = "unknown",
             **kwargs) -> TuningResult:
        if problem_size and device:
            cached = self.cache.get(kernel_type, problem_size, device)
            if cached:
                metrics = self._benchmark_config(cached, *args, **kwargs)
                if metrics:
                    return TuningResult(best_config=cached, metrics=metrics, problem_size=problem_size, device=device)
        results = []
        best = None
        for config in self.all_configs:
            m = self._benchmark_config(config, *args, **kwargs)
            if m is None:
                continue
            results.append((dict(config), m))
            if best is None or m.latency_ms < best[1].latency_ms:
                best = (dict(config), m)
        if best is None:
            raise TuningFailedError(f"No valid configuration found for {kernel_type}", problem_size=problem_size,
                                    configs_tried=len(self.all_configs))
        if problem_size and device:
            self.cache.set(kernel_type, problem_size, device, best[0])
        return TuningResult(best_config=best[0], metrics=best[1], all_results=results, problem_size=problem_size,
                            device=device)

    def get_cached_config(self, problem_size: Tuple[int, ...], device: str, kernel_type: str = "unknown"):
        return self.cache.get(kernel_type, problem_size, device)

    def clear_cache(self) -> None:
        self.cache.clear()


def compute_gemm_metrics(M: int, N: int, K: int, latency_ms: float, peak_tflops: float = B200_PEAK_TFLOPS_BF16,
                         peak_bandwidth_gbps: float = B200_PEAK_HBM_GBPS, dtype_bytes: int = 2) -> KernelMetrics:
    """Metrics of one M x N x K GEMM (2*M*N*K flops, A + B + C bytes)."""
    s = latency_ms / 1e3
    tflops = 2.0 * M * N * K / s / 1e12 if s > 0 else 0.0
    gbps = (M * K + K * N + M * N) * dtype_bytes / s / 1e9 if s > 0 else 0.0
    return KernelMetrics(latency_ms=latency_ms, throughput_tflops=tflops, bandwidth_gbps=gbps,
                         bandwidth_utilization=100.0 * tflops / peak_tflops if peak_tflops else 0.0)


def compute_elementwise_metrics(num_elements: int, latency_ms: float, bytes_per_element: int = 4,
                                peak_bandwidth_gbps: float = B200_PEAK_HBM_GBPS) -> KernelMetrics:
    """Metrics of a memory-bound op moving bytes_per_element per element."""
    s = latency_ms / 1e3
    gbps = num_elements * bytes_per_element / s / 1e9 if s > 0 else 0.0
    return KernelMetrics(latency_ms=latency_ms, throughput_tflops=0.0, bandwidth_gbps=gbps,
                         bandwidth_utilization=100.0 * gbps / peak_bandwidth_gbps if peak_bandwidth_gbps else 0.0)
