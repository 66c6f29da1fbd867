"""Functional API (same names and signatures as the reference's triton_ops/api.py:36-195)."""

from typing import Literal, Optional

import torch

from triton_ops.kernels.fp8_gemm import FP8Linear
from triton_ops.kernels.fp8_gemm import fp8_gemm as _fp8_gemm
from triton_ops.kernels.fp8_quantize import dequantize_fp8 as _dequantize_fp8
from triton_ops.kernels.fp8_quantize import quantize_fp8 as _quantize_fp8
from triton_ops.kernels.gated_mlp import FusedGatedMLP
from triton_ops.kernels.gated_mlp import fused_gated_mlp as _fused_gated_mlp
from triton_ops.kernels.rmsnorm_rope import FusedRMSNormRoPE
from triton_ops.kernels.rmsnorm_rope import fused_rmsnorm_rope as _fused_rmsnorm_rope


def fused_rmsnorm_rope(
    x: torch.Tensor,
    weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    eps: float = 1e-6,
    num_heads: Optional[int] = None,
) -> torch.Tensor:
    """RMSNorm (``x * rsqrt(mean(x^2) + eps) * weight``) then rotate-half RoPE, in one kernel.

    x: [batch, seq_len, hidden]; weight: [hidden]; cos/sin: [seq_len, head_dim].
    """
    return _fused_rmsnorm_rope(x, weight, cos, sin, eps, num_heads)


def fused_gated_mlp(
    x: torch.Tensor,
    gate_weight: torch.Tensor,
    up_weight: torch.Tensor,
    activation: Literal["silu", "gelu", "gelu_tanh"] = "silu",
) -> torch.Tensor:
    """``gate_proj(x) * activation(up_proj(x))`` with both projections in one kernel."""
    return _fused_gated_mlp(x, gate_weight, up_weight, activation)


def fp8_gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    a_scale: Optional[torch.Tensor] = None,
    b_scale: Optional[torch.Tensor] = None,
    output_dtype: torch.dtype = torch.float16,
) -> torch.Tensor:
    """FP8 matrix product; float operands are quantized first (per-tensor scale)."""
    return _fp8_gemm(a, b, a_scale, b_scale, output_dtype)


def quantize_fp8(
    tensor: torch.Tensor,
    scale: Optional[torch.Tensor] = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-tensor 8-bit quantization; returns (codes, scale)."""
    return _quantize_fp8(tensor, scale)


def dequantize_fp8(
    tensor: torch.Tensor,
    scale: torch.Tensor,
    output_dtype: torch.dtype = torch.float16,
) -> torch.Tensor:
    """Inverse of :func:`quantize_fp8`."""
    return _dequantize_fp8(tensor, scale, output_dtype)


__all__ = [
    "fused_rmsnorm_rope",
    "fused_gated_mlp",
    "fp8_gemm",
    "quantize_fp8",
    "dequantize_fp8",
    "FusedRMSNormRoPE",
    "FusedGatedMLP",
    "FP8Linear",
]
