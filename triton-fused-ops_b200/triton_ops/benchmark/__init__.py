"""Benchmark helpers (reference-compatible API; timing with CUDA events)."""

from triton_ops.benchmark.correctness import CorrectnessVerifier
from triton_ops.benchmark.report import PerformanceReport
from triton_ops.benchmark.suite import BenchmarkSuite

__all__ = ["BenchmarkSuite", "CorrectnessVerifier", "PerformanceReport"]
