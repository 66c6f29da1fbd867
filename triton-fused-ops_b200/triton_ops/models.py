"""Data models: tensor specs, op input specs, metrics and the FP8 format.

Field names, defaults and methods follow the reference (triton_ops/models.py).
``FP8Format.compute_scale`` is on the hot path of ``quantize_fp8``; here it is
one device reduction plus the scale computed on the GPU, with no host
synchronisation, and it returns the same fp32 value the reference computes on
the host (``fp32(448 / double(max|x|))``, 1.0 when the tensor is all zeros).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Literal, Optional, Tuple

import torch


@dataclass
class TensorSpec:
    """Shape / dtype / device / contiguity of a tensor argument."""

    shape: Tuple[int, ...]
    dtype: torch.dtype
    device: str = "cuda"
    contiguous: bool = True

    def validate(self, tensor: torch.Tensor) -> bool:
        """True if `tensor` matches this specification."""
        if tuple(tensor.shape) != tuple(self.shape):
            return False
        if tensor.dtype != self.dtype:
            return False
        if self.device == "cuda" and not tensor.is_cuda:
            return False
        if self.contiguous and not tensor.is_contiguous():
            return False
        return True

    def create_tensor(self, fill_value: Optional[float] = None) -> torch.Tensor:
        """A tensor matching the spec: filled with `fill_value`, else N(0, 1)."""
        if fill_value is not None:
            return torch.full(self.shape, fill_value, dtype=self.dtype, device=self.device)
        return torch.randn(self.shape, dtype=self.dtype, device=self.device)


@dataclass
class RMSNormRoPEInput:
    """Input specification of fused RMSNorm + RoPE."""

    x: TensorSpec
    weight: TensorSpec
    cos: TensorSpec
    sin: TensorSpec
    eps: float = 1e-6

    @classmethod
    def from_shapes(
        cls,
        batch_size: int,
        seq_len: int,
        hidden_dim: int,
        head_dim: int,
        dtype: torch.dtype = torch.float16,
        device: str = "cuda",
        eps: float = 1e-6,
    ) -> "RMSNormRoPEInput":
        return cls(
            x=TensorSpec((batch_size, seq_len, hidden_dim), dtype, device),
            weight=TensorSpec((hidden_dim,), dtype, device),
            cos=TensorSpec((seq_len, head_dim), dtype, device),
            sin=TensorSpec((seq_len, head_dim), dtype, device),
            eps=eps,
        )


@dataclass
class GatedMLPInput:
    """Input specification of the fused gated MLP."""

    x: TensorSpec
    gate_weight: TensorSpec
    up_weight: TensorSpec
    activation: Literal["silu", "gelu"] = "silu"

    @classmethod
    def from_shapes(
        cls,
        batch_size: int,
        seq_len: int,
        hidden_dim: int,
        intermediate_dim: int,
        activation: Literal["silu", "gelu"] = "silu",
        dtype: torch.dtype = torch.float16,
        device: str = "cuda",
    ) -> "GatedMLPInput":
        return cls(
            x=TensorSpec((batch_size, seq_len, hidden_dim), dtype, device),
            gate_weight=TensorSpec((intermediate_dim, hidden_dim), dtype, device),
            up_weight=TensorSpec((intermediate_dim, hidden_dim), dtype, device),
            activation=activation,
        )


@dataclass
class FP8GEMMInput:
    """Input specification of the FP8 GEMM."""

    a: TensorSpec
    b: TensorSpec
    a_scale: TensorSpec
    b_scale: TensorSpec
    output_dtype: torch.dtype = torch.float16

    @classmethod
    def from_shapes(
        cls,
        M: int,
        N: int,
        K: int,
        output_dtype: torch.dtype = torch.float16,
        device: str = "cuda",
    ) -> "FP8GEMMInput":
        fp8_dtype = getattr(torch, "float8_e4m3fn", torch.uint8)
        return cls(
            a=TensorSpec((M, K), fp8_dtype, device),
            b=TensorSpec((K, N), fp8_dtype, device),
            a_scale=TensorSpec((1,), torch.float32, device),
            b_scale=TensorSpec((1,), torch.float32, device),
            output_dtype=output_dtype,
        )


@dataclass
class KernelMetrics:
    """Timing and throughput of one kernel execution."""

    latency_ms: float
    throughput_tflops: float
    bandwidth_gbps: float
    bandwidth_utilization: float

    def __str__(self) -> str:
        return (
            f"Latency: {self.latency_ms:.3f} ms, "
            f"Throughput: {self.throughput_tflops:.2f} TFLOPS, "
            f"Bandwidth: {self.bandwidth_gbps:.1f} GB/s ({self.bandwidth_utilization:.1f}%)"
        )


@dataclass
class TuningResult:
    """Outcome of a configuration search."""

    best_config: Dict[str, Any]
    metrics: KernelMetrics
    all_results: List[Tuple[Dict[str, Any], KernelMetrics]] = field(default_factory=list)
    problem_size: Optional[Tuple[int, ...]] = None
    device: Optional[str] = None

    def __str__(self) -> str:
        config_str = ", ".join(f"{k}={v}" for k, v in self.best_config.items())
        return f"Best config: {{{config_str}}}\n{self.metrics}"


@dataclass
class FP8Format:
    """FP8 E4M3 format constants and per-tensor scale helpers."""

    exponent_bits: int = 4
    mantissa_bits: int = 3
    max_value: float = 448.0
    min_normal: float = 2**-6

    @staticmethod
    def compute_scale(tensor: torch.Tensor) -> torch.Tensor:
        """Per-tensor quantize multiplier ``448 / max|x|`` as a 0-dim fp32 CUDA tensor.

        Computed by the native amax kernel (reference: triton_ops/models.py:282-299);
        the result is bit-identical to the reference's host computation and no
        host synchronisation happens.
        """
        from triton_ops import _lib
        from triton_ops.validation import _check_cuda, _check_dtype, SUPPORTED_DTYPES_FLOAT

        _check_cuda(tensor, "tensor")
        _check_dtype(tensor, "tensor", SUPPORTED_DTYPES_FLOAT)
        t = tensor.contiguous()
        n = t.numel()
        scale = torch.empty((), dtype=torch.float32, device=t.device)
        lib = _lib.load()
        ws_bytes = lib.tfo_fp8_scale_workspace_bytes(n)
        ws = _lib.workspace(ws_bytes, t.device)
        _lib.call(
            "tfo_fp8_compute_scale",
            t.data_ptr(), n, _lib.dtype_code(t.dtype), scale.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_of(t),
        )
        return scale

    @staticmethod
    def compute_scale_per_channel(tensor: torch.Tensor, dim: int = 0) -> torch.Tensor:
        """Per-channel multipliers ``448 / max|x|`` along `dim` (1 where the max is 0).

        Reducing over the last dimension of a contiguous CUDA tensor (``dim=-1``:
        per token of activations, per output channel of an ``[out, in]`` weight)
        runs the library's kernel (``tfo_fp8_compute_scale_rows``), which
        rounds like the torch expression below (``448.0 / t`` is
        ``t.reciprocal() * 448`` in the tensor's dtype) and returns the same
        values, dtype and ``[..., 1]`` shape.
        """
        if (tensor.is_cuda and tensor.is_contiguous() and tensor.dim() >= 1 and tensor.numel() > 0
                and dim in (-1, tensor.dim() - 1) and tensor.dtype in (torch.float16, torch.bfloat16, torch.float32)):
            from triton_ops import _lib

            cols = tensor.shape[-1]
            out = torch.empty(*tensor.shape[:-1], 1, dtype=torch.float32, device=tensor.device)
            _lib.call("tfo_fp8_compute_scale_rows", tensor.data_ptr(), tensor.numel() // cols, cols,
                      _lib.dtype_code(tensor.dtype), out.data_ptr(), _lib.stream_of(tensor))
            return out if tensor.dtype == torch.float32 else out.to(tensor.dtype)
        max_abs = tensor.abs().amax(dim=dim, keepdim=True)
        max_abs = torch.where(max_abs == 0, torch.ones_like(max_abs), max_abs)
        return FP8Format.max_value / max_abs

    @staticmethod
    def is_in_range(tensor: torch.Tensor, scale: torch.Tensor) -> bool:
        """True if every element of ``tensor * scale`` is within +-448."""
        scaled = tensor * scale
        return bool(scaled.abs().max() <= FP8Format.max_value)
