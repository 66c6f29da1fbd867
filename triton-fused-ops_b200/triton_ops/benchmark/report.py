"""Benchmark records and text/JSON reports (API of the reference's report module)."""

import json
from dataclasses import asdict, dataclass, field
from datetime import datetime
from typing import Any, Dict, List, Optional

from triton_ops.models import KernelMetrics


@dataclass
class BenchmarkResult:
    kernel_name: str
    problem_size: tuple
    config: Dict[str, Any]
    metrics: KernelMetrics
    correctness: bool
    timestamp: Optional[str] = None

    def __post_init__(self):
        if self.timestamp is None:
            self.timestamp = datetime.now().isoformat()


@dataclass
class ComparisonResult:
    kernel_name: str
    problem_size: tuple
    triton_metrics: KernelMetrics
    baseline_metrics: KernelMetrics
    speedup: float
    correctness: bool


class PerformanceReport:
    def __init__(self, title: str = "Fused Operators Benchmark Report (B200)"):
        self.title = title
        self.results: List[BenchmarkResult] = []
        self.comparisons: List[ComparisonResult] = []
        self.metadata: Dict[str, Any] = {}

    def add_result(self, result: BenchmarkResult) -> None:
        self.results.append(result)

    def add_comparison(self, comparison: ComparisonResult) -> None:
        self.comparisons.append(comparison)

    def set_metadata(self, key: str, value: Any) -> None:
        self.metadata[key] = value

    def generate_text_report(self) -> str:
        lines = [self.title, "=" * len(self.title)]
        for k, v in self.metadata.items():
            lines.append(f"{k}: {v}")
        if self.results:
            lines.append("")
            lines.append("Results")
            for r in self.results:
                status = "PASS" if r.correctness else "FAIL"
                lines.append(f"  {r.kernel_name} {r.problem_size} [{status}] {r.metrics}")
        if self.comparisons:
            lines.append("")
            lines.append("Comparisons")
            for c in self.comparisons:
                lines.append(f"  {c.kernel_name} {c.problem_size}: speedup {c.speedup:.2f}x "
                             f"({'match' if c.correctness else 'MISMATCH'})")
        return "\n".join(lines)

    def generate_json_report(self) -> str:
        def conv(obj):
            d = asdict(obj)
            d["problem_size"] = list(d["problem_size"])
            return d

        return json.dumps({"title": self.title, "metadata": self.metadata,
                           "results": [conv(r) for r in self.results],
                           "comparisons": [conv(c) for c in self.comparisons]}, indent=2, default=str)

    def save(self, filepath: str, format: str = "text") -> None:
        with open(filepath, "w") as f:
            f.write(self.generate_json_report() if format == "json" else self.generate_text_report())
